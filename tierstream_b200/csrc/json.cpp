#include "json.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "errors.hpp"

namespace tsb {

Json Json::number(int64_t v) {
  Json j = number(v < 0 ? uint64_t(0) - uint64_t(v) : uint64_t(v));  // the magnitude, exact for INT64_MIN too
  j.neg = v < 0;
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

constexpr size_t kMaxDepth = 64;

bool is_digit(char c) { return c >= '0' && c <= '9'; }

// 0..15 for a hex digit, -1 otherwise
int hex_value(char c) {
  if (is_digit(c)) return c - '0';
  const char l = char(c | 0x20);
  return l >= 'a' && l <= 'f' ? l - 'a' + 10 : -1;
}

// Appends code point `cp` (<= 0x10FFFF) as UTF-8: a lead byte carrying the top bits, then 6 bits per continuation byte.
void put_utf8(std::string& out, uint32_t cp) {
  static const uint8_t kLead[4] = {0x00, 0xC0, 0xE0, 0xF0};
  const int tail = cp < 0x80 ? 0 : cp < 0x800 ? 1 : cp < 0x10000 ? 2 : 3;
  out += char(kLead[tail] | (cp >> (6 * tail)));
  for (int k = tail - 1; k >= 0; --k) out += char(0x80 | ((cp >> (6 * k)) & 0x3F));
}

// RFC 8259 text -> Json without recursion: containers still open are kept on an explicit stack, each with the key
// its next member goes under. Errors are SS_E_DESC naming the byte offset.
class Reader {
 public:
  explicit Reader(const std::string& text) : at_(text.data()), begin_(text.data()), end_(text.data() + text.size()) {}

  Json document() {
    Json j = next_value();
    skip_space();
    if (at_ != end_) error("trailing data");
    return j;
  }

 private:
  struct Open {
    Json value;       // an Object or an Array
    std::string key;  // (objects) the key of the member being read
  };
  const char* at_;
  const char* begin_;
  const char* end_;

  [[noreturn]] void error(const std::string& what) const {
    fail(SS_E_DESC, "json: " + what + " at offset " + std::to_string(size_t(at_ - begin_)));
  }
  char peek() const { return at_ < end_ ? *at_ : '\0'; }
  bool eat(char c) {
    if (peek() != c || at_ == end_) return false;
    ++at_;
    return true;
  }
  void skip_space() {
    while (at_ < end_ && (*at_ == ' ' || *at_ == '\n' || *at_ == '\r' || *at_ == '\t')) ++at_;
  }
  static char closer(const Json& c) { return c.kind == Json::Object ? '}' : ']'; }

  // A member's key and its ':' (the next value is the member's).
  void member_key(Open& o) {
    skip_space();
    if (!eat('"')) error("expected a key");
    o.key = string_body();
    if (o.value.obj.count(o.key)) error("duplicate key \"" + o.key + "\"");
    skip_space();
    if (!eat(':')) error("expected ':'");
  }

  Json next_value() {
    std::vector<Open> open;
    for (;;) {
      skip_space();
      Json done;
      const char c = peek();
      if (at_ < end_ && (c == '{' || c == '[')) {
        if (open.size() >= kMaxDepth) error("nesting deeper than 64");
        ++at_;
        open.push_back(Open{c == '{' ? Json::object() : Json::array(), {}});
        skip_space();
        if (!eat(closer(open.back().value))) {
          if (c == '{') member_key(open.back());
          continue;  // its first member's value
        }
        done = std::move(open.back().value);  // empty
        open.pop_back();
      } else {
        done = scalar();
      }
      // `done` goes into the innermost open container; each container that closes here is itself done
      for (;;) {
        if (open.empty()) return done;
        Open& o = open.back();
        const bool is_object = o.value.kind == Json::Object;
        if (is_object) o.value.obj.emplace(std::move(o.key), std::move(done));
        else o.value.arr.push_back(std::move(done));
        skip_space();
        if (eat(',')) {
          if (is_object) member_key(o);
          break;
        }
        if (!eat(closer(o.value))) error(is_object ? "expected ',' or '}'" : "expected ',' or ']'");
        done = std::move(o.value);
        open.pop_back();
      }
    }
  }

  Json scalar() {
    if (at_ == end_) error("unexpected end");
    if (eat('"')) return Json::string(string_body());
    for (const char* w : {"true", "false", "null"}) {
      const size_t n = std::strlen(w);
      if (size_t(end_ - at_) >= n && std::memcmp(at_, w, n) == 0) {
        at_ += n;
        return w[0] == 'n' ? Json{} : Json::boolean(w[0] == 't');
      }
    }
    return number();
  }

  // After the opening quote, through the closing one: plain runs are appended whole, escapes one at a time.
  std::string string_body() {
    std::string out;
    for (;;) {
      const char* run = at_;
      while (at_ < end_ && *at_ != '"' && *at_ != '\\' && uint8_t(*at_) >= 0x20) ++at_;
      out.append(run, size_t(at_ - run));
      if (at_ == end_) error("unterminated string");
      const char c = *at_++;
      if (c == '"') return out;
      if (c != '\\') error("control character in a string");
      escape(out);
    }
  }

  void escape(std::string& out) {
    static const char kPairs[] = "\"\"\\\\//b\bf\fn\nr\rt\t";  // (escape letter, character) pairs
    if (at_ == end_) error("unterminated escape");
    const char e = *at_++;
    for (const char* p = kPairs; *p; p += 2)
      if (p[0] == e) {
        out += p[1];
        return;
      }
    if (e != 'u') error("bad escape");
    uint32_t cp = code_unit();
    if (cp >= 0xDC00 && cp < 0xE000) error("lone surrogate");
    if (cp >= 0xD800 && cp < 0xDC00) {  // a high surrogate: its low half must follow as another \u escape
      if (!(end_ - at_ >= 2 && at_[0] == '\\' && at_[1] == 'u')) error("lone surrogate");
      at_ += 2;
      const uint32_t low = code_unit();
      if (low < 0xDC00 || low >= 0xE000) error("bad surrogate pair");
      cp = 0x10000 + (((cp & 0x3FF) << 10) | (low & 0x3FF));
    }
    put_utf8(out, cp);
  }

  uint32_t code_unit() {
    if (end_ - at_ < 4) error("short \\u escape");
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const int h = hex_value(*at_++);
      if (h < 0) error("bad \\u escape");
      v = v * 16 + uint32_t(h);
    }
    return v;
  }

  // -?(0|[1-9][0-9]*)(\.[0-9]+)?([eE][+-]?[0-9]+)? ; an integer form that fits 64 bits keeps its exact magnitude
  Json number() {
    const char* start = at_;
    const bool negative = eat('-');
    auto digits = [&](const char* what) {
      if (!is_digit(peek())) error(what);
      while (is_digit(peek())) ++at_;
    };
    const char* int_begin = at_;
    digits("bad number");
    if (*int_begin == '0' && at_ - int_begin > 1) {
      at_ = int_begin + 1;
      error("leading zero");
    }
    const char* int_end = at_;
    bool integral = true;
    if (eat('.')) {
      integral = false;
      digits("bad fraction");
    }
    if (peek() == 'e' || peek() == 'E') {
      ++at_;
      integral = false;
      if (peek() == '+' || peek() == '-') ++at_;
      digits("bad exponent");
    }
    Json j = Json::number(std::strtod(std::string(start, at_).c_str(), nullptr));
    if (!integral) return j;
    uint64_t mag = 0;
    for (const char* p = int_begin; p < int_end; ++p)
      if (__builtin_mul_overflow(mag, uint64_t(10), &mag) || __builtin_add_overflow(mag, uint64_t(*p - '0'), &mag))
        return j;  // beyond 64 bits: the double only
    j.is_int = true;
    j.u = mag;
    j.neg = negative && mag != 0;
    return j;
  }
};

// Canonical text: object keys in sorted order (std::map), no whitespace, integers exact, other numbers integral
// below 9e15 as integers, else %.17g; strings escape '"', '\\', \n, \r, \t and other control bytes as \u00XX.
class Writer {
 public:
  std::string out;

  void value(const Json& j) {
    switch (j.kind) {
      case Json::Null: out += "null"; return;
      case Json::Bool: out += j.b ? "true" : "false"; return;
      case Json::Number: number(j); return;
      case Json::String: text(j.s); return;
      case Json::Array: {
        char sep = '[';
        for (const Json& v : j.arr) {
          out += sep;
          sep = ',';
          value(v);
        }
        out += j.arr.empty() ? "[]" : "]";
        return;
      }
      case Json::Object: {
        char sep = '{';
        for (const auto& kv : j.obj) {
          out += sep;
          sep = ',';
          text(kv.first);
          out += ':';
          value(kv.second);
        }
        out += j.obj.empty() ? "{}" : "}";
        return;
      }
    }
  }

 private:
  void number(const Json& j) {
    if (j.is_int) {
      if (j.neg) out += '-';
      out += std::to_string(j.u);
      return;
    }
    if (std::isfinite(j.d) && std::fabs(j.d) < 9e15 && std::trunc(j.d) == j.d) {
      out += std::to_string(int64_t(j.d));
      return;
    }
    char buf[40];
    std::snprintf(buf, sizeof buf, "%.17g", j.d);
    out += buf;
  }

  void text(const std::string& s) {
    out += '"';
    for (const char ch : s) {
      const uint8_t c = uint8_t(ch);
      const char* esc = c == '"' ? "\\\"" : c == '\\' ? "\\\\" : c == '\n' ? "\\n" : c == '\r' ? "\\r"
                        : c == '\t' ? "\\t" : nullptr;
      if (esc) {
        out += esc;
      } else if (c < 0x20) {
        char buf[8];
        std::snprintf(buf, sizeof buf, "\\u%04x", c);
        out += buf;
      } else {
        out += ch;
      }
    }
    out += '"';
  }
};

}  // namespace

Json json_parse(const std::string& text) { return Reader(text).document(); }

std::string json_write(const Json& j) {
  Writer w;
  w.value(j);
  return std::move(w.out);
}

uint64_t json_u64(const Json& j, const std::string& where) {
  require(j.kind == Json::Number && j.is_int && !j.neg, SS_E_DESC, where + ": expected an unsigned 64-bit integer");
  return j.u;
}

int64_t json_i64(const Json& j, const std::string& where) {
  const uint64_t limit = uint64_t(INT64_MAX) + (j.neg ? 1 : 0);
  require(j.kind == Json::Number && j.is_int && j.u <= limit, SS_E_DESC, where + ": expected a 64-bit integer");
  return j.neg ? int64_t(uint64_t(0) - j.u) : int64_t(j.u);
}

double json_f64(const Json& j, const std::string& where) {
  require(j.kind == Json::Number, SS_E_DESC, where + ": expected a number");
  if (!j.is_int) return j.d;
  return j.neg ? -double(j.u) : double(j.u);
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
