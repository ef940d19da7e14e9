// abi_generate.cc -- the text layer of rpg_engine_generate.
//
// Behaviour follows the reference host code so a request produces the same
// prompt ids and the same response structure:
//  * tokenizer  src/tokenizer.cc: GPT-2 byte-level alphabet, Qwen2
//               pre-tokenizer split, merges by rank (leftmost on ties), greedy
//               longest-first match of CONTROL/USER_DEFINED specials, decode
//               without skipping specials;
//  * ChatML     src/chat_template.cc:85-206 (Qwen3's template: tools block,
//               <think> handling after the last user query, tool responses
//               grouped into one user turn, generation prompt);
//  * output     src/tool_parser.cc:125-178 (strip control markers, <think>
//               blocks, <tool_call>{json}</tool_call> extraction);
//  * driver     src/engine.cc:429-615 (longest common prefix with the cached
//               ids, capacity check before touching the cache, stop ids = eos,
//               <|im_end|> and single-token stop strings, top_k 0 / top_p 0.95,
//               finish_reason rules, usage).
#include "abi_generate.h"

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <unordered_map>

#include "common.h"

namespace rpgb {

namespace {

#include "unicode_ranges.inc"

template <size_t N>
bool InRanges(const uint32_t (&r)[N][2], uint32_t cp) {
  size_t lo = 0, hi = N;
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid][0]) {
      hi = mid;
    } else if (cp > r[mid][1]) {
      lo = mid + 1;
    } else {
      return true;
    }
  }
  return false;
}
bool IsLetter(uint32_t c) { return InRanges(kLetterRanges, c); }
bool IsNumber(uint32_t c) { return InRanges(kNumberRanges, c); }
bool IsSpace(uint32_t c) { return InRanges(kSpaceRanges, c); }
bool IsNl(uint32_t c) { return c == '\r' || c == '\n'; }

// UTF-8 decode; an invalid sequence yields U+FFFD consuming one byte.
uint32_t DecodeAt(const std::string& s, size_t i, int* len) {
  const unsigned char b0 = static_cast<unsigned char>(s[i]);
  if (b0 < 0x80) {
    *len = 1;
    return b0;
  }
  int n = 0;
  uint32_t cp = 0;
  if ((b0 & 0xE0) == 0xC0) {
    n = 2;
    cp = b0 & 0x1F;
  } else if ((b0 & 0xF0) == 0xE0) {
    n = 3;
    cp = b0 & 0x0F;
  } else if ((b0 & 0xF8) == 0xF0) {
    n = 4;
    cp = b0 & 0x07;
  } else {
    *len = 1;
    return 0xFFFD;
  }
  if (i + n > s.size()) {
    *len = 1;
    return 0xFFFD;
  }
  for (int k = 1; k < n; ++k) {
    const unsigned char b = static_cast<unsigned char>(s[i + k]);
    if ((b & 0xC0) != 0x80) {
      *len = 1;
      return 0xFFFD;
    }
    cp = (cp << 6) | (b & 0x3F);
  }
  const uint32_t min_cp[5] = {0, 0, 0x80, 0x800, 0x10000};
  if (cp < min_cp[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) {
    *len = 1;
    return 0xFFFD;
  }
  *len = n;
  return cp;
}

void PutUtf8(uint32_t cp, std::string* out) {
  if (cp < 0x80) {
    out->push_back(static_cast<char>(cp));
  } else if (cp < 0x800) {
    out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  } else {
    out->push_back(static_cast<char>(0xF0 | (cp >> 18)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
    out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
  }
}

// GPT-2 byte-level alphabet.
struct ByteMap {
  uint32_t to_cp[256];
  int16_t to_byte[324];
  ByteMap() {
    std::fill(std::begin(to_byte), std::end(to_byte), int16_t(-1));
    uint32_t extra = 0;
    for (int b = 0; b < 256; ++b) {
      const bool direct = (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || b >= 174;
      to_cp[b] = direct ? static_cast<uint32_t>(b) : 256 + extra++;
      to_byte[to_cp[b]] = static_cast<int16_t>(b);
    }
  }
  int Byte(uint32_t cp) const { return cp < 324 ? to_byte[cp] : -1; }
};
const ByteMap& Bytes() {
  static const ByteMap m;
  return m;
}

struct Cp {
  uint32_t cp;
  size_t off;
};

std::vector<Cp> Cps(const std::string& s) {
  std::vector<Cp> v;
  v.reserve(s.size());
  for (size_t i = 0; i < s.size();) {
    int len = 1;
    const uint32_t c = DecodeAt(s, i, &len);
    v.push_back({c, i});
    i += static_cast<size_t>(len);
  }
  return v;
}

// Length (in code points) of the Qwen2 pre-tokenizer match starting at p:
//   (?i:'s|'t|'re|'ve|'m|'ll|'d) | [^\r\n\p{L}\p{N}]?\p{L}+ | \p{N}
//   | ?[^\s\p{L}\p{N}]+[\r\n]* | \s*[\r\n]+ | \s+(?!\S) | \s+
size_t SplitLen(const std::vector<Cp>& c, size_t p) {
  const size_t n = c.size();
  const uint32_t c0 = c[p].cp;
  if (c0 == '\'' && p + 1 < n) {
    const uint32_t a = c[p + 1].cp | 0x20;
    const bool ascii_letter = (c[p + 1].cp >= 'a' && c[p + 1].cp <= 'z') || (c[p + 1].cp >= 'A' && c[p + 1].cp <= 'Z');
    if (ascii_letter) {
      if (a == 's' || a == 't' || a == 'm' || a == 'd') return 2;
      if (p + 2 < n) {
        const uint32_t b = c[p + 2].cp | 0x20;
        const bool b_letter = (c[p + 2].cp >= 'a' && c[p + 2].cp <= 'z') || (c[p + 2].cp >= 'A' && c[p + 2].cp <= 'Z');
        if (b_letter && (((a == 'r' || a == 'v') && b == 'e') || (a == 'l' && b == 'l'))) return 3;
      }
    }
  }
  {
    size_t q = p;
    if (!IsNl(c0) && !IsLetter(c0) && !IsNumber(c0)) ++q;
    size_t r = q;
    while (r < n && IsLetter(c[r].cp)) ++r;
    if (r > q) return r - p;
    if (q != p) {  // the optional prefix did not lead to letters: retry without it
      r = p;
      while (r < n && IsLetter(c[r].cp)) ++r;
      if (r > p) return r - p;
    }
  }
  if (IsNumber(c0)) return 1;
  {
    size_t q = c0 == ' ' ? p + 1 : p;
    size_t r = q;
    while (r < n && !IsSpace(c[r].cp) && !IsLetter(c[r].cp) && !IsNumber(c[r].cp)) ++r;
    if (r == q && q != p) {  // " " alone did not start a run: retry without the space
      q = p;
      r = p;
      while (r < n && !IsSpace(c[r].cp) && !IsLetter(c[r].cp) && !IsNumber(c[r].cp)) ++r;
    }
    if (r > q) {
      while (r < n && IsNl(c[r].cp)) ++r;
      return r - p;
    }
  }
  if (IsSpace(c0)) {
    size_t e = p;
    while (e < n && IsSpace(c[e].cp)) ++e;
    size_t last_nl = SIZE_MAX;
    for (size_t i = p; i < e; ++i) {
      if (IsNl(c[i].cp)) last_nl = i;
    }
    if (last_nl != SIZE_MAX) return last_nl - p + 1;
    if (e == n) return e - p;
    if (e - p >= 2) return e - 1 - p;
    return e - p;
  }
  return 1;
}

std::string TrimAscii(const std::string& s) {
  size_t b = 0, e = s.size();
  auto sp = [](char ch) { return ch == ' ' || ch == '\t' || ch == '\r' || ch == '\n' || ch == '\f' || ch == '\v'; };
  while (b < e && sp(s[b])) ++b;
  while (e > b && sp(s[e - 1])) --e;
  return s.substr(b, e - b);
}

bool StartsWith(const std::string& s, const std::string& p) { return s.compare(0, p.size(), p) == 0 && s.size() >= p.size(); }
bool EndsWith(const std::string& s, const std::string& p) {
  return s.size() >= p.size() && s.compare(s.size() - p.size(), p.size(), p) == 0;
}
std::string TrimNl(const std::string& s, bool left, bool right) {
  size_t b = 0, e = s.size();
  if (left) {
    while (b < e && s[b] == '\n') ++b;
  }
  if (right) {
    while (e > b && s[e - 1] == '\n') --e;
  }
  return s.substr(b, e - b);
}

}  // namespace

// ------------------------------------------------------------------ tokenizer

struct Tokenizer::Impl {
  std::unordered_map<std::string, int32_t> id_of;
  std::unordered_map<std::string, int32_t> rank;  // "left\x1Fright" -> merge rank
  std::vector<std::pair<std::string, int32_t>> specials;  // longest first
};

Tokenizer::Tokenizer(const GgufFile& g) : impl_(std::make_shared<Impl>()) {
  tokens_ = g.GetStrArray("tokenizer.ggml.tokens");
  RPGB_CHECK(!tokens_.empty(), "the GGUF has no tokenizer.ggml.tokens");
  const std::vector<int64_t> ty = g.GetIntArray("tokenizer.ggml.token_type");
  types_.assign(tokens_.size(), 1);
  if (!ty.empty()) {
    RPGB_CHECK(ty.size() == tokens_.size(), "token_type has %zu entries for %zu tokens", ty.size(), tokens_.size());
    for (size_t i = 0; i < ty.size(); ++i) types_[i] = static_cast<int32_t>(ty[i]);
  }
  for (size_t i = 0; i < tokens_.size(); ++i) impl_->id_of.emplace(tokens_[i], static_cast<int32_t>(i));
  const std::vector<std::string> merges = g.GetStrArray("tokenizer.ggml.merges");
  RPGB_CHECK(!merges.empty(), "the GGUF has no tokenizer.ggml.merges (byte-level BPE needs them)");
  for (size_t i = 0; i < merges.size(); ++i) {
    const size_t sp = merges[i].find(' ');
    RPGB_CHECK(sp != std::string::npos, "merge %zu has no separator", i);
    std::string key = merges[i].substr(0, sp);
    key.push_back('\x1F');
    key.append(merges[i], sp + 1, std::string::npos);
    impl_->rank.emplace(std::move(key), static_cast<int32_t>(i));
  }
  for (size_t i = 0; i < tokens_.size(); ++i) {
    if (types_[i] == 3 || types_[i] == 4) impl_->specials.emplace_back(tokens_[i], static_cast<int32_t>(i));
  }
  std::stable_sort(impl_->specials.begin(), impl_->specials.end(),
                   [](const auto& a, const auto& b) { return a.first.size() > b.first.size(); });
}

int32_t Tokenizer::IdOf(const std::string& tok) const {
  const auto it = impl_->id_of.find(tok);
  return it == impl_->id_of.end() ? -1 : it->second;
}

std::vector<int32_t> Tokenizer::Encode(const std::string& text, bool parse_special) const {
  std::vector<int32_t> out;
  auto encode_plain = [&](const std::string& t) {
    const std::vector<Cp> cps = Cps(t);
    size_t p = 0;
    while (p < cps.size()) {
      size_t len = SplitLen(cps, p);
      if (len == 0) len = 1;
      const size_t end = p + len;
      const size_t b0 = cps[p].off, b1 = end < cps.size() ? cps[end].off : t.size();
      // byte-level symbols of the piece
      std::vector<std::string> sym;
      for (size_t i = b0; i < b1; ++i) {
        std::string s;
        PutUtf8(Bytes().to_cp[static_cast<unsigned char>(t[i])], &s);
        sym.push_back(std::move(s));
      }
      std::string key;
      while (sym.size() > 1) {
        int best = -1, best_rank = INT_MAX;
        for (size_t i = 0; i + 1 < sym.size(); ++i) {
          key = sym[i];
          key.push_back('\x1F');
          key += sym[i + 1];
          const auto it = impl_->rank.find(key);
          if (it != impl_->rank.end() && it->second < best_rank) {
            best_rank = it->second;
            best = static_cast<int>(i);
          }
        }
        if (best < 0) break;
        sym[best] += sym[best + 1];
        sym.erase(sym.begin() + best + 1);
      }
      for (const std::string& s : sym) {
        const int32_t id = IdOf(s);
        if (id >= 0) {
          out.push_back(id);
          continue;
        }
        // not in the vocabulary: fall back to its byte tokens
        for (const Cp& c : Cps(s)) {
          const int b = Bytes().Byte(c.cp);
          RPGB_CHECK(b >= 0, "symbol %s is neither a token nor a byte", s.c_str());
          std::string bs;
          PutUtf8(Bytes().to_cp[b], &bs);
          const int32_t bid = IdOf(bs);
          RPGB_CHECK(bid >= 0, "byte 0x%02X has no token", b);
          out.push_back(bid);
        }
      }
      p = end;
    }
  };
  size_t i = 0, plain = 0;
  const size_t n = text.size();
  while (i < n) {
    int32_t hit = -1;
    size_t hit_len = 0;
    if (parse_special) {
      for (const auto& sp : impl_->specials) {
        if (sp.first.size() <= n - i && text.compare(i, sp.first.size(), sp.first) == 0) {
          hit = sp.second;
          hit_len = sp.first.size();
          break;
        }
      }
    }
    if (hit >= 0) {
      if (i > plain) encode_plain(text.substr(plain, i - plain));
      out.push_back(hit);
      i += hit_len;
      plain = i;
    } else {
      ++i;
    }
  }
  if (n > plain) encode_plain(text.substr(plain));
  return out;
}

std::string Tokenizer::Decode(const std::vector<int32_t>& ids) const {
  std::string out;
  for (const int32_t id : ids) {
    if (id < 0 || static_cast<size_t>(id) >= tokens_.size()) continue;
    for (const Cp& c : Cps(tokens_[static_cast<size_t>(id)])) {
      const int b = Bytes().Byte(c.cp);
      if (b >= 0) {
        out.push_back(static_cast<char>(b));
      } else {
        PutUtf8(c.cp, &out);
      }
    }
  }
  return out;
}

// ------------------------------------------------------------------ ChatML

namespace {

struct ToolCall {
  std::string name, arguments;
};
struct Message {
  std::string role, content, reasoning;
  bool has_reasoning = false;
  std::vector<ToolCall> calls;
};

bool Truthy(const Json& j) {
  switch (j.type()) {
    case Json::Type::kNull: return false;
    case Json::Type::kBool: return j.AsBool();
    case Json::Type::kNumber: return j.AsDouble() != 0.0;
    case Json::Type::kString: return !j.AsString().empty();
    default: return j.size() != 0;
  }
}

std::vector<Message> ParseMessages(const Json& arr) {
  std::vector<Message> out;
  for (size_t i = 0; i < arr.size(); ++i) {
    const Json& m = arr.At(i);
    Message msg;
    if (m.Get("role").IsString()) msg.role = m.Get("role").AsString();
    if (m.Get("content").IsString()) msg.content = m.Get("content").AsString();
    if (m.Get("reasoning_content").IsString()) {
      msg.has_reasoning = true;
      msg.reasoning = m.Get("reasoning_content").AsString();
    }
    const Json& tcs = m.Get("tool_calls");
    for (size_t k = 0; k < tcs.size(); ++k) {
      const Json& tc = tcs.At(k);
      const Json& src = tc.Get("function").IsObject() ? tc.Get("function") : tc;
      ToolCall c;
      if (src.Get("name").IsString()) c.name = src.Get("name").AsString();
      const Json& a = src.Get("arguments");
      c.arguments = a.IsString() ? a.AsString() : a.DumpPython();
      msg.calls.push_back(std::move(c));
    }
    out.push_back(std::move(msg));
  }
  return out;
}

// Qwen3's chat template text (the model was trained on exactly these strings).
const char kToolsHead[] =
    "# Tools\n\nYou may call one or more functions to assist with the user query.\n\n"
    "You are provided with function signatures within <tools></tools> XML tags:\n<tools>";
const char kToolsTail[] =
    "\n</tools>\n\nFor each function call, return a json object with function name and arguments within "
    "<tool_call></tool_call> XML tags:\n<tool_call>\n{\"name\": <function-name>, \"arguments\": "
    "<args-json-object>}\n</tool_call><|im_end|>\n";

std::string RenderChatml(const std::vector<Message>& msgs, const Json& tools, bool enable_thinking) {
  std::string out;
  const bool first_sys = !msgs.empty() && msgs[0].role == "system";
  if (Truthy(tools)) {
    out += "<|im_start|>system\n";
    if (first_sys) out += msgs[0].content + "\n\n";
    out += kToolsHead;
    for (size_t i = 0; i < tools.size(); ++i) out += "\n" + tools.At(i).DumpPython();
    out += kToolsTail;
  } else if (first_sys) {
    out += "<|im_start|>system\n" + msgs[0].content + "<|im_end|>\n";
  }
  const int64_t n = static_cast<int64_t>(msgs.size());
  int64_t last_query = n - 1;
  for (int64_t i = n - 1; i >= 0; --i) {
    const Message& m = msgs[static_cast<size_t>(i)];
    if (m.role == "user" && !(StartsWith(m.content, "<tool_response>") && EndsWith(m.content, "</tool_response>"))) {
      last_query = i;
      break;
    }
  }
  for (int64_t i = 0; i < n; ++i) {
    const Message& m = msgs[static_cast<size_t>(i)];
    std::string content = m.content;
    if (m.role == "user" || (m.role == "system" && i != 0)) {
      out += "<|im_start|>" + m.role + "\n" + content + "<|im_end|>\n";
    } else if (m.role == "assistant") {
      std::string reasoning;
      if (m.has_reasoning) {
        reasoning = m.reasoning;
      } else if (content.find("</think>") != std::string::npos) {
        std::string before = TrimNl(content.substr(0, content.find("</think>")), false, true);
        const size_t o = before.rfind("<think>");
        if (o != std::string::npos) before = before.substr(o + 7);
        reasoning = TrimNl(before, true, false);
        content = TrimNl(content.substr(content.rfind("</think>") + 8), true, false);
      }
      out += "<|im_start|>assistant\n";
      if (i > last_query && (i == n - 1 || !reasoning.empty())) {
        out += "<think>\n" + TrimNl(reasoning, true, true) + "\n</think>\n\n" + TrimNl(content, true, false);
      } else {
        out += content;
      }
      for (size_t k = 0; k < m.calls.size(); ++k) {
        if ((k == 0 && !content.empty()) || k != 0) out += "\n";
        out += "<tool_call>\n{\"name\": \"" + m.calls[k].name + "\", \"arguments\": " + m.calls[k].arguments +
               "}\n</tool_call>";
      }
      out += "<|im_end|>\n";
    } else if (m.role == "tool") {
      if (i == 0 || msgs[static_cast<size_t>(i - 1)].role != "tool") out += "<|im_start|>user";
      out += "\n<tool_response>\n" + content + "\n</tool_response>";
      if (i == n - 1 || msgs[static_cast<size_t>(i + 1)].role != "tool") out += "<|im_end|>\n";
    }
  }
  out += "<|im_start|>assistant\n";
  if (!enable_thinking) out += "<think>\n\n</think>\n\n";
  return out;
}

// ------------------------------------------------------------------ output parsing

struct ParsedCall {
  std::string name;
  Json arguments;
  bool ok = false;
};
struct Parsed {
  std::string text;
  std::vector<ParsedCall> calls;
  bool open_call = false, open_think = false;
};

ParsedCall ParseCall(const std::string& body) {
  ParsedCall c;
  std::string err;
  const Json j = Json::Parse(TrimAscii(body), &err);
  if (!j.IsObject()) return c;
  if (j.Get("name").IsString()) c.name = j.Get("name").AsString();
  const Json& a = j.Get("arguments");
  if (a.IsString()) {
    std::string e2;
    const Json inner = Json::Parse(a.AsString(), &e2);
    if (inner.IsObject()) c.arguments = inner;
  } else if (a.IsObject()) {
    c.arguments = a;
  }
  c.ok = !c.name.empty() && c.arguments.IsObject();
  return c;
}

void EraseAll(std::string* s, const std::string& marker) {
  for (size_t p = s->find(marker); p != std::string::npos; p = s->find(marker, p)) s->erase(p, marker.size());
}

Parsed ParseOutput(const std::string& raw) {
  Parsed out;
  std::string w = raw;
  const std::string start = "<|im_start|>";
  for (size_t p = w.find(start); p != std::string::npos; p = w.find(start, p)) {
    size_t end = p + start.size();
    for (const char* role : {"system", "user", "assistant", "tool"}) {
      const size_t rl = std::strlen(role);
      if (w.compare(end, rl, role) == 0 && end + rl < w.size() && w[end + rl] == '\n') {
        end += rl + 1;
        break;
      }
    }
    w.erase(p, end - p);
  }
  EraseAll(&w, "<|im_end|>");
  EraseAll(&w, "<|endoftext|>");
  for (;;) {
    const size_t b = w.find("<think>");
    if (b == std::string::npos) break;
    const size_t e = w.find("</think>", b + 7);
    if (e == std::string::npos) {
      w.erase(b);
      out.open_think = true;
      break;
    }
    w.erase(b, e + 8 - b);
  }
  size_t pos = 0;
  std::string text;
  for (;;) {
    const size_t b = w.find("<tool_call>", pos);
    if (b == std::string::npos) break;
    text.append(w, pos, b - pos);
    const size_t body = b + 11;
    const size_t e = w.find("</tool_call>", body);
    if (e == std::string::npos) {
      out.calls.push_back(ParseCall(w.substr(body)));
      out.open_call = true;
      pos = w.size();
      break;
    }
    out.calls.push_back(ParseCall(w.substr(body, e - body)));
    pos = e + 12;
  }
  text.append(w, pos, std::string::npos);
  out.text = TrimAscii(text);
  return out;
}

void AddStop(const Tokenizer& tok, const std::string& s, std::vector<int32_t>* ids) {
  if (s.empty()) return;
  const int32_t direct = tok.IdOf(s);
  if (direct >= 0) {
    ids->push_back(direct);
    return;
  }
  const std::vector<int32_t> enc = tok.Encode(s, false);
  if (enc.size() == 1) {
    ids->push_back(enc[0]);
  } else {
    RPGB_WARN("stop string '%s' is not a single token (%zu tokens); ignored", s.c_str(), enc.size());
  }
}

}  // namespace

std::string RenderRequestPrompt(const Json& req) {
  const std::vector<Message> msgs = ParseMessages(req.Get("messages"));
  RPGB_CHECK(!msgs.empty(), "messages is empty: at least one message is required");
  const Json tools = req.Get("tools").IsArray() ? req.Get("tools") : Json::Array();
  const bool thinking = req.Get("enable_thinking").AsBool(true);
  return RenderChatml(msgs, tools, thinking);
}

Json ParseOutputJson(const std::string& raw) {
  const Parsed p = ParseOutput(raw);
  Json o = Json::Object();
  o.Set("text", Json::Str(p.text));
  Json calls = Json::Array();
  for (const ParsedCall& pc : p.calls) {
    Json one = Json::Object();
    one.Set("name", Json::Str(pc.name));
    one.Set("arguments", pc.ok ? pc.arguments : Json());
    calls.Push(one);
  }
  o.Set("tool_calls", calls);
  o.Set("unterminated_think", Json::Bool(p.open_think));
  o.Set("unterminated_tool_call", Json::Bool(p.open_call));
  return o;
}

std::string RunGenerate(const GenerateState& st, const Json& req) {
  Session& sess = *st.sess;
  const Tokenizer& tok = *st.tok;
  const ModelMeta& c = sess.model().meta();

  const std::string prompt = RenderRequestPrompt(req);
  std::vector<int32_t> ids = tok.Encode(prompt, true);
  if (c.add_bos && c.bos_id >= 0) ids.insert(ids.begin(), c.bos_id);
  const int64_t total = static_cast<int64_t>(ids.size());
  RPGB_CHECK(total > 0, "the rendered prompt encodes to no tokens");

  std::vector<int32_t>& cached = *st.cached_ids;
  RPGB_CHECK(static_cast<int64_t>(cached.size()) == sess.len(), "internal state mismatch: cached ids %zu, kv len %lld",
             cached.size(), static_cast<long long>(sess.len()));
  int64_t lcp = 0;
  while (lcp < static_cast<int64_t>(cached.size()) && lcp < total && cached[lcp] == ids[lcp]) ++lcp;
  if (lcp == total) lcp = total - 1;  // forward at least one position

  int32_t max_tokens = static_cast<int32_t>(req.Get("max_tokens").AsInt(st.max_tokens));
  if (max_tokens <= 0) max_tokens = st.max_tokens;
  float temperature = static_cast<float>(req.Get("temperature").AsDouble(st.temperature));
  if (temperature < 0.0f) temperature = 0.0f;
  if (temperature > 2.0f) temperature = 2.0f;
  const uint64_t seed = static_cast<uint64_t>(req.Get("seed").AsInt(static_cast<int64_t>(st.seed)));
  RPGB_CHECK(total + max_tokens + 4 <= sess.max_seq(),
             "sequence too long: prompt %lld + generation %d + margin 4 exceed the session capacity %lld "
             "(raise session_json.max_seq or call session_reset)",
             static_cast<long long>(total), max_tokens, static_cast<long long>(sess.max_seq()));

  sess.SetLen(lcp);
  cached.resize(static_cast<size_t>(lcp));
  try {
    sess.Prefill(ids.data() + lcp, total - lcp, nullptr);
    cached.assign(ids.begin(), ids.end());
  } catch (...) {
    sess.SetLen(0);
    cached.clear();
    throw;
  }

  std::vector<int32_t> stop_ids;
  if (c.eos_id >= 0) stop_ids.push_back(c.eos_id);
  const int32_t im_end = tok.IdOf("<|im_end|>");
  if (im_end >= 0 && std::find(stop_ids.begin(), stop_ids.end(), im_end) == stop_ids.end()) stop_ids.push_back(im_end);
  const Json& rstop = req.Get("stop");
  for (size_t i = 0; i < rstop.size(); ++i) {
    if (rstop.At(i).IsString()) AddStop(tok, rstop.At(i).AsString(), &stop_ids);
  }
  for (const std::string& s : *st.stop) AddStop(tok, s, &stop_ids);

  SampleOpts opt;
  opt.temperature = temperature;
  opt.top_k = 0;
  opt.top_p = 0.95f;
  std::vector<int32_t> gen(static_cast<size_t>(max_tokens));
  int n = 0;
  try {
    n = sess.Generate(opt, seed, max_tokens, stop_ids.data(), static_cast<int32_t>(stop_ids.size()), gen.data(),
                      nullptr);
  } catch (...) {
    // a failed decode leaves the cache at a length the cached ids do not
    // describe: start the session over, so the next request prefills again
    // (src/engine.cc:531-537 does the same after a failed prefill)
    sess.SetLen(0);
    cached.clear();
    throw;
  }
  gen.resize(static_cast<size_t>(n));
  cached.insert(cached.end(), gen.begin(), gen.end());

  const Parsed parsed = ParseOutput(tok.Decode(gen));
  std::string finish;
  if (!parsed.calls.empty()) {
    finish = "tool_calls";
  } else if (parsed.open_call || parsed.open_think) {
    finish = "length";
  } else if (static_cast<int32_t>(gen.size()) >= max_tokens &&
             (gen.empty() || std::find(stop_ids.begin(), stop_ids.end(), gen.back()) == stop_ids.end())) {
    finish = "length";
  } else {
    finish = "stop";
  }
  Json resp = Json::Object();
  resp.Set("text", Json::Str(parsed.text));
  Json calls = Json::Array();
  for (const ParsedCall& pc : parsed.calls) {
    Json one = Json::Object();
    one.Set("name", Json::Str(pc.name));
    one.Set("arguments", pc.ok ? pc.arguments : Json());
    calls.Push(one);
  }
  resp.Set("tool_calls", calls);
  resp.Set("finish_reason", Json::Str(finish));
  Json usage = Json::Object();
  usage.Set("prompt_tokens", Json::Number(static_cast<double>(total)));
  usage.Set("completion_tokens", Json::Number(static_cast<double>(gen.size())));
  resp.Set("usage", usage);
  return resp.Dump();
}

}  // namespace rpgb
