// json.h -- minimal JSON value, parser and serializer for the public ABI.
//
// The reference ships its own JSON DOM (src/json.h); the ABI only needs to read
// config / request objects and write response objects, so this is a small
// independent implementation: UTF-8 strings, \uXXXX escapes with surrogate
// pairs, numbers as double (integers kept exact up to 2^53).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace rpgb {

class Json {
 public:
  enum class Type { kNull, kBool, kNumber, kString, kArray, kObject };

  Json() = default;
  static Json Bool(bool b);
  static Json Number(double d);
  static Json IntLiteral(double d);  // a number written without '.' or exponent
  static Json Str(const std::string& s);
  static Json Array();
  static Json Object();

  // Parses `text`; on failure returns null and sets *err.
  static Json Parse(const std::string& text, std::string* err);
  std::string Dump() const;
  // Python json.dumps style (", " and ": " separators, integer literals kept
  // as integers, floats in shortest round-trip form) -- the form in which tool
  // schemas appear inside the chat prompt.
  std::string DumpPython() const;

  Type type() const { return type_; }
  bool IsNull() const { return type_ == Type::kNull; }
  bool IsBool() const { return type_ == Type::kBool; }
  bool IsNumber() const { return type_ == Type::kNumber; }
  bool IsIntLiteral() const { return type_ == Type::kNumber && int_lit_; }
  bool IsString() const { return type_ == Type::kString; }
  bool IsArray() const { return type_ == Type::kArray; }
  bool IsObject() const { return type_ == Type::kObject; }

  bool AsBool(bool def = false) const { return IsBool() ? b_ : def; }
  double AsDouble(double def = 0.0) const { return IsNumber() ? d_ : def; }
  int64_t AsInt(int64_t def = 0) const { return IsNumber() ? static_cast<int64_t>(d_) : def; }
  const std::string& AsString() const { return s_; }

  // object access; missing keys return a shared null
  bool Has(const std::string& k) const { return IsObject() && obj_->count(k) != 0; }
  const Json& Get(const std::string& k) const;
  Json& Set(const std::string& k, Json v);
  // array access
  size_t size() const;
  const Json& At(size_t i) const;
  void Push(Json v);
  const std::vector<std::pair<std::string, Json>>& Items() const;  // object in insertion order

 private:
  Type type_ = Type::kNull;
  bool int_lit_ = false;
  bool b_ = false;
  double d_ = 0.0;
  std::string s_;
  std::shared_ptr<std::vector<Json>> arr_;
  std::shared_ptr<std::map<std::string, Json>> obj_;
  std::shared_ptr<std::vector<std::pair<std::string, Json>>> order_;
};

void JsonEscape(const std::string& s, std::string* out);

}  // namespace rpgb
