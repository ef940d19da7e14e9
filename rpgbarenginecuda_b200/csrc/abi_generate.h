// abi_generate.h -- text layer behind rpg_engine_generate (tokenizer, ChatML,
// tool-call parsing) and the generate driver.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "engine.h"
#include "gguf.h"
#include "json.h"

namespace rpgb {

class Tokenizer {
 public:
  explicit Tokenizer(const GgufFile& g);
  int32_t vocab_size() const { return static_cast<int32_t>(tokens_.size()); }
  int32_t IdOf(const std::string& tok) const;
  std::vector<int32_t> Encode(const std::string& text, bool parse_special) const;
  std::string Decode(const std::vector<int32_t>& ids) const;

 private:
  std::vector<std::string> tokens_;
  std::vector<int32_t> types_;
  struct Impl;
  std::shared_ptr<Impl> impl_;
};

struct GenerateState {
  Session* sess;
  const Tokenizer* tok;
  std::vector<int32_t>* cached_ids;
  int32_t max_tokens;
  float temperature;
  uint64_t seed;
  const std::vector<std::string>* stop;
};

// Runs one rpg_engine_generate request; returns the response JSON text.
std::string RunGenerate(const GenerateState& st, const Json& req);

// The ChatML prompt rpg_engine_generate renders for a request (its messages,
// tools and enable_thinking keys).
std::string RenderRequestPrompt(const Json& req);

// The model-output parse rpg_engine_generate applies to the decoded text:
// {text, tool_calls: [{name, arguments (object or null)}],
// unterminated_think, unterminated_tool_call}.
Json ParseOutputJson(const std::string& raw);

}  // namespace rpgb
