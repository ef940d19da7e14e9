// ref_text_shim.cc -- extern "C" bridge into the reference's host text layer,
// compiled from its own sources by oracle/Makefile into oracle/_ref/.
//
// TEST INFRASTRUCTURE ONLY: the tests compare the engine's text layer with
// these outputs byte for byte.  Each entry calls the function the reference's
// rpg_engine_generate calls (src/engine.cc:429-615):
//   Tokenizer::FromGguf / Encode / Decode   src/tokenizer.cc:132-200, 314, 353
//   ParseMessages / ParseTools / RenderChatml  src/chat_template.cc:85-206
//   ParseModelOutput                         src/tool_parser.cc:125-178
// Returned strings are malloc'd; free them with reft_free.
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "chat_template.h"
#include "gguf.h"
#include "json.h"
#include "tokenizer.h"
#include "tool_parser.h"

namespace {

thread_local std::string g_err;

struct TextHandle {
  rpg::GgufFile gguf;
  rpg::Tokenizer tok;
};

char* Dup(const std::string& s) {
  char* p = static_cast<char*>(std::malloc(s.size() + 1));
  std::memcpy(p, s.data(), s.size());
  p[s.size()] = '\0';
  return p;
}

}  // namespace

extern "C" {

const char* reft_last_error() { return g_err.c_str(); }

void reft_free(char* p) { std::free(p); }

void* reft_open(const char* gguf_path) {
  try {
    auto h = std::make_unique<TextHandle>();
    h->gguf = rpg::GgufFile::Open(gguf_path);
    h->tok = rpg::Tokenizer::FromGguf(h->gguf);
    return h.release();
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

void reft_close(void* h) { delete static_cast<TextHandle*>(h); }

// Token ids of text; returns the count (written up to cap), -1 on error.
int64_t reft_encode(void* h, const char* text, int64_t len, int parse_special, int32_t* out, int64_t cap) {
  try {
    const auto ids = static_cast<TextHandle*>(h)->tok.Encode(std::string(text, static_cast<size_t>(len)),
                                                              parse_special != 0);
    for (size_t i = 0; i < ids.size() && static_cast<int64_t>(i) < cap; ++i) out[i] = ids[i];
    return static_cast<int64_t>(ids.size());
  } catch (const std::exception& e) {
    g_err = e.what();
    return -1;
  }
}

// Bytes of the decoded ids (may hold NUL bytes: *out_len is the length).
char* reft_decode(void* h, const int32_t* ids, int64_t n, int skip_special, int64_t* out_len) {
  try {
    const std::string s = static_cast<TextHandle*>(h)->tok.Decode(std::vector<int32_t>(ids, ids + n), skip_special != 0);
    *out_len = static_cast<int64_t>(s.size());
    return Dup(s);
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

// The prompt rpg_engine_generate renders for a request's messages and tools.
char* reft_render(const char* messages_json, const char* tools_json, int add_generation_prompt, int enable_thinking) {
  try {
    std::string err;
    const rpg::Json msgs = rpg::Json::Parse(messages_json, &err);
    const rpg::Json tools_in = tools_json != nullptr ? rpg::Json::Parse(tools_json, &err) : rpg::Json();
    rpg::ChatTemplateOptions opt;
    opt.add_generation_prompt = add_generation_prompt != 0;
    opt.enable_thinking = enable_thinking != 0;
    return Dup(rpg::RenderChatml(rpg::ParseMessages(msgs), rpg::ParseTools(tools_in), opt));
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

// ParseModelOutput of raw model text, as JSON: {text, reasoning, tool_calls:
// [{name, arguments_raw, arguments, ok}], unterminated_think,
// unterminated_tool_call}.
char* reft_parse(const char* raw, int64_t len) {
  try {
    const rpg::ParsedOutput p = rpg::ParseModelOutput(std::string(raw, static_cast<size_t>(len)));
    rpg::Json o = rpg::Json::Object();
    o["text"] = p.text;
    o["reasoning"] = p.reasoning;
    rpg::Json calls = rpg::Json::Array();
    for (const auto& c : p.tool_calls) {
      rpg::Json j = rpg::Json::Object();
      j["name"] = c.name;
      j["arguments_raw"] = c.arguments_raw;
      j["arguments"] = c.arguments.Dump();
      j["ok"] = c.ok;
      calls.PushBack(j);
    }
    o["tool_calls"] = calls;
    o["unterminated_think"] = p.unterminated_think;
    o["unterminated_tool_call"] = p.unterminated_tool_call;
    return Dup(o.Dump());
  } catch (const std::exception& e) {
    g_err = e.what();
    return nullptr;
  }
}

}  // extern "C"
