#include "json.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "errors.hpp"

namespace tsb {

Json Json::number(int64_t v) {
  Json j;
  j.kind = Number;
  j.is_int = true;
  j.neg = v < 0;
  j.u = v < 0 ? uint64_t(0) - uint64_t(v) : uint64_t(v);
  j.d = double(v);
  return j;
}

Json Json::number(double v) {
  Json j;
  j.kind = Number;
  j.d = v;
  return j;
}

namespace {

struct Parser {
  const std::string& t;
  size_t i = 0;
  int depth = 0;

  [[noreturn]] void bad(const std::string& what) const {
    fail(SS_E_DESC, "json: " + what + " at offset " + std::to_string(i));
  }
  void ws() {
    while (i < t.size() && (t[i] == ' ' || t[i] == '\t' || t[i] == '\n' || t[i] == '\r')) ++i;
  }
  bool lit(const char* w) {
    size_t n = 0;
    while (w[n]) ++n;
    if (t.compare(i, n, w) != 0) return false;
    i += n;
    return true;
  }
  static void utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
      out += char(cp);
    } else if (cp < 0x800) {
      out += char(0xC0 | (cp >> 6));
      out += char(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      out += char(0xE0 | (cp >> 12));
      out += char(0x80 | ((cp >> 6) & 0x3F));
      out += char(0x80 | (cp & 0x3F));
    } else {
      out += char(0xF0 | (cp >> 18));
      out += char(0x80 | ((cp >> 12) & 0x3F));
      out += char(0x80 | ((cp >> 6) & 0x3F));
      out += char(0x80 | (cp & 0x3F));
    }
  }
  uint32_t hex4() {
    if (i + 4 > t.size()) bad("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = t[i++];
      v <<= 4;
      if (c >= '0' && c <= '9') v |= uint32_t(c - '0');
      else if (c >= 'a' && c <= 'f') v |= uint32_t(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') v |= uint32_t(c - 'A' + 10);
      else bad("bad \\u escape");
    }
    return v;
  }
  std::string str() {
    if (t[i] != '"') bad("expected a string");
    ++i;
    std::string out;
    for (;;) {
      if (i >= t.size()) bad("unterminated string");
      const char c = t[i++];
      if (c == '"') break;
      if (uint8_t(c) < 0x20) bad("control character in a string");
      if (c != '\\') {
        out += c;
        continue;
      }
      if (i >= t.size()) bad("unterminated escape");
      const char e = t[i++];
      switch (e) {
        case '"': out += '"'; break;
        case '\\': out += '\\'; break;
        case '/': out += '/'; break;
        case 'b': out += '\b'; break;
        case 'f': out += '\f'; break;
        case 'n': out += '\n'; break;
        case 'r': out += '\r'; break;
        case 't': out += '\t'; break;
        case 'u': {
          uint32_t cp = hex4();
          if (cp >= 0xD800 && cp < 0xDC00) {
            if (!(i + 1 < t.size() && t[i] == '\\' && t[i + 1] == 'u')) bad("lone surrogate");
            i += 2;
            const uint32_t lo = hex4();
            if (lo < 0xDC00 || lo >= 0xE000) bad("bad surrogate pair");
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          } else if (cp >= 0xDC00 && cp < 0xE000) {
            bad("lone surrogate");
          }
          utf8(out, cp);
          break;
        }
        default: bad("bad escape");
      }
    }
    return out;
  }
  Json num() {
    const size_t start = i;
    bool neg = false;
    if (t[i] == '-') {
      neg = true;
      ++i;
    }
    if (i >= t.size() || !(t[i] >= '0' && t[i] <= '9')) bad("bad number");
    if (t[i] == '0' && i + 1 < t.size() && t[i + 1] >= '0' && t[i + 1] <= '9') bad("leading zero");
    bool integer = true, overflow = false;
    uint64_t mag = 0;
    while (i < t.size() && t[i] >= '0' && t[i] <= '9') {
      const uint64_t dgt = uint64_t(t[i] - '0');
      if (mag > (UINT64_MAX - dgt) / 10) overflow = true;
      else mag = mag * 10 + dgt;
      ++i;
    }
    if (i < t.size() && t[i] == '.') {
      integer = false;
      ++i;
      if (i >= t.size() || !(t[i] >= '0' && t[i] <= '9')) bad("bad fraction");
      while (i < t.size() && t[i] >= '0' && t[i] <= '9') ++i;
    }
    if (i < t.size() && (t[i] == 'e' || t[i] == 'E')) {
      integer = false;
      ++i;
      if (i < t.size() && (t[i] == '+' || t[i] == '-')) ++i;
      if (i >= t.size() || !(t[i] >= '0' && t[i] <= '9')) bad("bad exponent");
      while (i < t.size() && t[i] >= '0' && t[i] <= '9') ++i;
    }
    Json j;
    j.kind = Json::Number;
    j.d = std::strtod(t.substr(start, i - start).c_str(), nullptr);
    if (integer && !overflow) {
      j.is_int = true;
      j.neg = neg && mag != 0;
      j.u = mag;
    }
    return j;
  }
  Json value() {
    ws();
    if (i >= t.size()) bad("unexpected end");
    const char c = t[i];
    if (c == '{') {
      if (++depth > 64) bad("nesting deeper than 64");
      ++i;
      Json j = Json::object();
      ws();
      if (i < t.size() && t[i] == '}') {
        ++i;
        --depth;
        return j;
      }
      for (;;) {
        ws();
        if (i >= t.size() || t[i] != '"') bad("expected a key");
        std::string k = str();
        ws();
        if (i >= t.size() || t[i] != ':') bad("expected ':'");
        ++i;
        if (j.obj.count(k)) bad("duplicate key \"" + k + "\"");
        j.obj.emplace(k, value());
        ws();
        if (i < t.size() && t[i] == ',') {
          ++i;
          continue;
        }
        if (i < t.size() && t[i] == '}') {
          ++i;
          break;
        }
        bad("expected ',' or '}'");
      }
      --depth;
      return j;
    }
    if (c == '[') {
      if (++depth > 64) bad("nesting deeper than 64");
      ++i;
      Json j = Json::array();
      ws();
      if (i < t.size() && t[i] == ']') {
        ++i;
        --depth;
        return j;
      }
      for (;;) {
        j.arr.push_back(value());
        ws();
        if (i < t.size() && t[i] == ',') {
          ++i;
          continue;
        }
        if (i < t.size() && t[i] == ']') {
          ++i;
          break;
        }
        bad("expected ',' or ']'");
      }
      --depth;
      return j;
    }
    if (c == '"') return Json::string(str());
    if (lit("true")) return Json::boolean(true);
    if (lit("false")) return Json::boolean(false);
    if (lit("null")) return Json{};
    return num();
  }
};

void write(const Json& j, std::string& o) {
  switch (j.kind) {
    case Json::Null: o += "null"; break;
    case Json::Bool: o += j.b ? "true" : "false"; break;
    case Json::Number:
      if (j.is_int) {
        if (j.neg) o += '-';
        o += std::to_string(j.u);
      } else if (std::isfinite(j.d) && j.d == std::floor(j.d) && std::fabs(j.d) < 9e15) {
        o += std::to_string(int64_t(j.d));
      } else {
        char buf[40];
        std::snprintf(buf, sizeof buf, "%.17g", j.d);
        o += buf;
      }
      break;
    case Json::String: {
      o += '"';
      for (unsigned char c : j.s) {
        if (c == '"') o += "\\\"";
        else if (c == '\\') o += "\\\\";
        else if (c == '\n') o += "\\n";
        else if (c == '\r') o += "\\r";
        else if (c == '\t') o += "\\t";
        else if (c < 0x20) {
          char buf[8];
          std::snprintf(buf, sizeof buf, "\\u%04x", c);
          o += buf;
        } else {
          o += char(c);
        }
      }
      o += '"';
      break;
    }
    case Json::Array:
      o += '[';
      for (size_t k = 0; k < j.arr.size(); ++k) {
        if (k) o += ',';
        write(j.arr[k], o);
      }
      o += ']';
      break;
    case Json::Object: {
      o += '{';
      bool first = true;
      for (const auto& kv : j.obj) {
        if (!first) o += ',';
        first = false;
        write(Json::string(kv.first), o);
        o += ':';
        write(kv.second, o);
      }
      o += '}';
      break;
    }
  }
}

}  // namespace

Json json_parse(const std::string& text) {
  Parser p{text};
  Json j = p.value();
  p.ws();
  if (p.i != text.size()) p.bad("trailing data");
  return j;
}

std::string json_write(const Json& j) {
  std::string o;
  write(j, o);
  return o;
}

uint64_t json_u64(const Json& j, const std::string& where) {
  require(j.kind == Json::Number && j.is_int && !j.neg, SS_E_DESC, where + ": expected an unsigned 64-bit integer");
  return j.u;
}

int64_t json_i64(const Json& j, const std::string& where) {
  require(j.kind == Json::Number && j.is_int && (j.neg ? j.u <= uint64_t(INT64_MAX) + 1 : j.u <= uint64_t(INT64_MAX)),
          SS_E_DESC, where + ": expected a 64-bit integer");
  return j.neg ? int64_t(uint64_t(0) - j.u) : int64_t(j.u);
}

double json_f64(const Json& j, const std::string& where) {
  require(j.kind == Json::Number, SS_E_DESC, where + ": expected a number");
  return j.is_int ? (j.neg ? -double(j.u) : double(j.u)) : j.d;
}

bool json_bool(const Json& j, const std::string& where) {
  require(j.kind == Json::Bool, SS_E_DESC, where + ": expected true or false");
  return j.b;
}

const std::string& json_str(const Json& j, const std::string& where) {
  require(j.kind == Json::String, SS_E_DESC, where + ": expected a string");
  return j.s;
}

}  // namespace tsb
