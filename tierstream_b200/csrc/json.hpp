// A small JSON value, parser and canonical writer (sorted keys, no whitespace) for the desc-v1 and plan-v1 documents.
// Integers keep their exact 64-bit value; duplicate keys, trailing data and nesting deeper than 64 are errors (SS_E_DESC).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace tsb {

struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  // numbers: exact integer when is_int (negative when neg, magnitude in u), else d
  bool is_int = false, neg = false;
  uint64_t u = 0;
  double d = 0;
  std::string s;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  static Json object() { Json j; j.kind = Object; return j; }
  static Json array() { Json j; j.kind = Array; return j; }
  static Json string(const std::string& v) { Json j; j.kind = String; j.s = v; return j; }
  static Json boolean(bool v) { Json j; j.kind = Bool; j.b = v; return j; }
  static Json number(uint64_t v) { Json j; j.kind = Number; j.is_int = true; j.u = v; j.d = double(v); return j; }
  static Json number(int64_t v);
  static Json number(double v);
  bool is_object() const { return kind == Object; }
  bool is_array() const { return kind == Array; }
  const Json* find(const std::string& k) const {
    if (kind != Object) return nullptr;
    auto it = obj.find(k);
    return it == obj.end() ? nullptr : &it->second;
  }
  Json& operator[](const std::string& k) { return obj[k]; }
  void push(const Json& v) { arr.push_back(v); }
};

Json json_parse(const std::string& text);
std::string json_write(const Json& j);
// Typed reads that fail with SS_E_DESC naming `where`.
uint64_t json_u64(const Json& j, const std::string& where);
int64_t json_i64(const Json& j, const std::string& where);
double json_f64(const Json& j, const std::string& where);
bool json_bool(const Json& j, const std::string& where);
const std::string& json_str(const Json& j, const std::string& where);

}  // namespace tsb
