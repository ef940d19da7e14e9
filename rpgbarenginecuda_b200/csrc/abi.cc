// abi.cc -- the ten-function public C ABI (include/rpg_engine.h).
//
// Same contract as the reference's src/engine.cc:
//  * no C++ exception crosses extern "C" (engine.cc:231-239): failures return
//    a negative value / NULL and the message goes to rpg_engine_last_error();
//  * handles are increasing integers, never reused (engine.cc:139-140);
//  * unloading a model cascades to its sessions (engine.cc:301-313);
//  * session_json keys max_seq / max_tokens / temperature (clamped to [0, 2]) /
//    seed / stop (engine.cc:315-391); config_json key context (engine.cc:262-268).
// Added: config_json "device" selects the GPU (default 0), so one process can
// serve sessions on several GPUs.
#include "../../include/rpg_engine.h"

#include <algorithm>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "abi_generate.h"
#include "common.h"
#include "engine.h"
#include "json.h"
#include "model.h"

namespace rpgb {
namespace {

constexpr const char* kVersion = "0.1.0";
constexpr int32_t kDefaultMaxTokens = 256;
constexpr float kMaxTemperature = 2.0f;

struct AbiModel {
  std::unique_ptr<Model> model;
  std::unique_ptr<Tokenizer> tok;
  int32_t max_pos = 0;
  std::vector<int32_t> sessions;
};

struct AbiSession {
  int32_t model = -1;
  std::unique_ptr<Session> sess;
  std::vector<int32_t> cached_ids;  // tokens whose K/V the cache holds
  int32_t max_tokens = kDefaultMaxTokens;
  std::vector<std::string> stop;
  float temperature = 0.0f;
  uint64_t seed = 0;
  int32_t max_seq = 0;
};

std::mutex g_mu;
std::map<int32_t, std::shared_ptr<AbiModel>> g_models;
std::map<int32_t, std::shared_ptr<AbiSession>> g_sessions;
int32_t g_next_model = 1;
int32_t g_next_session = 1;

char* Dup(const std::string& s) {
  char* b = new char[s.size() + 1];
  std::memcpy(b, s.data(), s.size());
  b[s.size()] = '\0';
  return b;
}

Json ParseConfig(const char* text, const char* what) {
  if (text == nullptr || *text == '\0') return Json::Object();
  std::string err;
  Json j = Json::Parse(text, &err);
  RPGB_CHECK(err.empty(), "%s is not valid JSON: %s", what, err.c_str());
  RPGB_CHECK(j.IsObject(), "%s must be a JSON object", what);
  return j;
}

std::shared_ptr<AbiModel> FindModel(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  const auto it = g_models.find(h);
  RPGB_CHECK(it != g_models.end(), "invalid model handle %d (unloaded?)", h);
  return it->second;
}

std::shared_ptr<AbiSession> FindSession(int32_t h) {
  std::lock_guard<std::mutex> lk(g_mu);
  const auto it = g_sessions.find(h);
  RPGB_CHECK(it != g_sessions.end(), "invalid session handle %d (destroyed?)", h);
  return it->second;
}

}  // namespace
}  // namespace rpgb

using namespace rpgb;

#define ABI_CATCH(ret)                                      \
  catch (const std::exception& e) {                         \
    SetLastError(e.what());                                 \
    return ret;                                             \
  }                                                         \
  catch (...) {                                             \
    SetLastError("unknown exception (not std::exception)"); \
    return ret;                                             \
  }

extern "C" {

const char* rpg_engine_version(void) { return kVersion; }

const char* rpg_engine_last_error(void) { return LastError(); }

int32_t rpg_engine_load_model(const char* model_path, const char* config_json) {
  try {
    SetLastError("");
    RPGB_CHECK(model_path != nullptr && *model_path != '\0', "model_path is empty");
    const Json cfg = ParseConfig(config_json, "config_json");
    const int device = static_cast<int>(cfg.Get("device").AsInt(0));
    auto e = std::make_shared<AbiModel>();
    // context: min(config, GGUF context_length); <= 0 means the GGUF value
    int32_t ctx = 1 << 30;
    if (cfg.Has("context")) ctx = static_cast<int32_t>(cfg.Get("context").AsInt(ctx));
    if (ctx <= 0) ctx = 1 << 30;
    e->model = Model::Load(model_path, device, ctx);
    e->max_pos = e->model->rope_positions();
    e->tok = std::make_unique<Tokenizer>(e->model->gguf());
    RPGB_CHECK(e->tok->vocab_size() == e->model->meta().vocab,
               "tokenizer vocab %d does not match the %d rows of token_embd", e->tok->vocab_size(),
               e->model->meta().vocab);
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next_model++;
    g_models[h] = e;
    return h;
  }
  ABI_CATCH(-1)
}

void rpg_engine_unload_model(int32_t model) {
  try {
    std::lock_guard<std::mutex> lk(g_mu);
    const auto it = g_models.find(model);
    if (it == g_models.end()) return;
    for (int32_t s : it->second->sessions) g_sessions.erase(s);
    g_models.erase(it);
  } catch (...) {
  }
}

int32_t rpg_engine_session_create(int32_t model, const char* session_json) {
  try {
    SetLastError("");
    auto m = FindModel(model);
    const Json cfg = ParseConfig(session_json, "session_json");
    auto s = std::make_shared<AbiSession>();
    s->model = model;
    s->max_seq = m->max_pos;
    if (cfg.Has("max_seq")) {
      const int64_t v = cfg.Get("max_seq").AsInt(m->max_pos);
      RPGB_CHECK(v > 0 && v <= m->max_pos, "session max_seq=%lld outside (0, %d]", static_cast<long long>(v),
                 m->max_pos);
      s->max_seq = static_cast<int32_t>(v);
    }
    if (cfg.Has("max_tokens")) {
      const int64_t v = cfg.Get("max_tokens").AsInt(kDefaultMaxTokens);
      s->max_tokens = static_cast<int32_t>(v > 0 ? v : kDefaultMaxTokens);
    }
    if (s->max_tokens >= s->max_seq) s->max_tokens = s->max_seq - 1;
    if (cfg.Has("temperature")) {
      float t = static_cast<float>(cfg.Get("temperature").AsDouble(0.0));
      if (t > kMaxTemperature) t = kMaxTemperature;
      s->temperature = t < 0.0f ? 0.0f : t;
    }
    if (cfg.Has("seed")) s->seed = static_cast<uint64_t>(cfg.Get("seed").AsInt(0));
    const Json& stop = cfg.Get("stop");
    for (size_t i = 0; i < stop.size(); ++i) {
      if (stop.At(i).IsString()) s->stop.push_back(stop.At(i).AsString());
    }
    s->sess = std::make_unique<Session>(m->model.get(), s->max_seq);
    std::lock_guard<std::mutex> lk(g_mu);
    const int32_t h = g_next_session++;
    g_sessions[h] = s;
    m->sessions.push_back(h);
    return h;
  }
  ABI_CATCH(-1)
}

void rpg_engine_session_destroy(int32_t session) {
  try {
    std::lock_guard<std::mutex> lk(g_mu);
    const auto it = g_sessions.find(session);
    if (it == g_sessions.end()) return;
    const auto mit = g_models.find(it->second->model);
    if (mit != g_models.end()) {
      auto& v = mit->second->sessions;
      v.erase(std::remove(v.begin(), v.end(), session), v.end());
    }
    g_sessions.erase(it);
  } catch (...) {
  }
}

int32_t rpg_engine_session_reset(int32_t session) {
  try {
    SetLastError("");
    auto s = FindSession(session);
    s->sess->SetLen(0);
    s->cached_ids.clear();
    return RPG_ENGINE_OK;
  }
  ABI_CATCH(-1)
}

char* rpg_engine_generate(int32_t session, const char* request_json) {
  try {
    SetLastError("");
    auto s = FindSession(session);
    auto m = FindModel(s->model);
    RPGB_CHECK(request_json != nullptr && *request_json != '\0', "request_json is empty");
    std::string err;
    const Json req = Json::Parse(request_json, &err);
    RPGB_CHECK(err.empty(), "request_json is not valid JSON: %s", err.c_str());
    RPGB_CHECK(req.IsObject(), "request_json must be a JSON object");
    GenerateState st{s->sess.get(), m->tok.get(), &s->cached_ids, s->max_tokens, s->temperature, s->seed,
                     &s->stop};
    return Dup(RunGenerate(st, req));
  }
  ABI_CATCH(nullptr)
}

void rpg_engine_free(char* buf) { delete[] buf; }

char* rpg_engine_model_info(int32_t model) {
  try {
    SetLastError("");
    auto m = FindModel(model);
    const ModelMeta& c = m->model->meta();
    Json o = Json::Object();
    o.Set("engine", Json::Str("rpg_engine_b200"));
    o.Set("engine_version", Json::Str(kVersion));
    o.Set("backend", Json::Str("cuda-sm_100a"));
    o.Set("arch", Json::Str(c.arch));
    o.Set("name", Json::Str(c.name));
    o.Set("n_layers", Json::Number(c.n_layers));
    o.Set("hidden", Json::Number(c.hidden));
    o.Set("n_heads", Json::Number(c.n_heads));
    o.Set("n_kv_heads", Json::Number(c.n_kv_heads));
    o.Set("head_dim", Json::Number(c.head_dim));
    o.Set("intermediate", Json::Number(c.ffn));
    o.Set("vocab", Json::Number(c.vocab));
    o.Set("context_length", Json::Number(c.context_length));
    o.Set("rope_theta", Json::Number(c.rope_theta));
    o.Set("tied_embeddings", Json::Bool(c.tied));
    o.Set("path", Json::Str(m->model->gguf().path()));
    o.Set("max_pos", Json::Number(m->max_pos));
    o.Set("default_max_seq", Json::Number(m->max_pos));
    o.Set("weight_bytes", Json::Number(static_cast<double>(c.weight_bytes)));
    {
      std::lock_guard<std::mutex> lk(g_mu);
      o.Set("sessions", Json::Number(static_cast<double>(m->sessions.size())));
    }
    o.Set("device_available", Json::Bool(true));
    o.Set("device", Json::Number(m->model->device()));
    o.Set("device_bytes", Json::Number(static_cast<double>(m->model->device_bytes())));
    return Dup(o.Dump());
  }
  ABI_CATCH(nullptr)
}

}  // extern "C"
