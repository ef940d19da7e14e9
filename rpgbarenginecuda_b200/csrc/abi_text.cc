// abi_text.cc -- extern "C" entries into the text layer of rpg_engine_generate
// (tokenizer, ChatML prompt, model-output parse), declared in
// include/rpg_b200.h.  They run the same functions rpg_engine_generate runs
// and need no GPU, so a host (or a test) can see the exact token ids and
// strings a request turns into.  Errors: NULL / -1 with the text in
// rpg_engine_last_error(); strings are new[]-allocated, freed with
// rpg_engine_free().
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/rpg_b200.h"
#include "abi_generate.h"
#include "common.h"
#include "gguf.h"
#include "json.h"

namespace {

struct TextHandle {
  rpgb::GgufFile gguf;
  std::unique_ptr<rpgb::Tokenizer> tok;
};

char* DupBytes(const std::string& s) {
  char* b = new char[s.size() + 1];
  std::memcpy(b, s.data(), s.size());
  b[s.size()] = '\0';
  return b;
}

rpgb::Json ParseArg(const char* text, const char* what) {
  std::string err;
  rpgb::Json j = rpgb::Json::Parse(text != nullptr ? text : "", &err);
  RPGB_CHECK(err.empty(), "%s is not valid JSON: %s", what, err.c_str());
  return j;
}

}  // namespace

#define TEXT_CATCH(ret)                        \
  catch (const std::exception& e) {            \
    rpgb::SetLastError(e.what());              \
    return ret;                                \
  }                                            \
  catch (...) {                                \
    rpgb::SetLastError("unknown exception");   \
    return ret;                                \
  }

extern "C" {

void* rpgb_text_open(const char* gguf_path) {
  try {
    RPGB_CHECK(gguf_path != nullptr && *gguf_path != '\0', "gguf_path is empty");
    auto h = std::make_unique<TextHandle>();
    h->gguf.Open(gguf_path);
    h->tok = std::make_unique<rpgb::Tokenizer>(h->gguf);
    return h.release();
  }
  TEXT_CATCH(nullptr)
}

void rpgb_text_close(void* h) { delete static_cast<TextHandle*>(h); }

int64_t rpgb_text_encode(void* h, const char* text, int64_t len, int32_t parse_special, int32_t* out, int64_t cap) {
  try {
    RPGB_CHECK(h != nullptr, "invalid text handle");
    RPGB_CHECK(len >= 0 && (text != nullptr || len == 0), "bad text");
    const std::vector<int32_t> ids =
        static_cast<TextHandle*>(h)->tok->Encode(std::string(text != nullptr ? text : "", static_cast<size_t>(len)),
                                                 parse_special != 0);
    for (size_t i = 0; i < ids.size() && static_cast<int64_t>(i) < cap; ++i) out[i] = ids[i];
    return static_cast<int64_t>(ids.size());
  }
  TEXT_CATCH(-1)
}

char* rpgb_text_decode(void* h, const int32_t* ids, int64_t n, int64_t* out_len) {
  try {
    RPGB_CHECK(h != nullptr, "invalid text handle");
    RPGB_CHECK(n >= 0 && (ids != nullptr || n == 0), "bad ids");
    const std::string s = static_cast<TextHandle*>(h)->tok->Decode(std::vector<int32_t>(ids, ids + n));
    if (out_len != nullptr) *out_len = static_cast<int64_t>(s.size());
    return DupBytes(s);
  }
  TEXT_CATCH(nullptr)
}

char* rpgb_text_render(const char* request_json) {
  try {
    return DupBytes(rpgb::RenderRequestPrompt(ParseArg(request_json, "request_json")));
  }
  TEXT_CATCH(nullptr)
}

char* rpgb_text_parse(const char* raw, int64_t len) {
  try {
    RPGB_CHECK(len >= 0 && (raw != nullptr || len == 0), "bad text");
    return DupBytes(rpgb::ParseOutputJson(std::string(raw != nullptr ? raw : "", static_cast<size_t>(len))).Dump());
  }
  TEXT_CATCH(nullptr)
}

}  // extern "C"
