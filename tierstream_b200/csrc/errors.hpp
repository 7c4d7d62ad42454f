// Library errors: a status from the C ABI's ss_status plus a message. Every C entry point maps them (capi.cpp).
#pragma once

#include <stdexcept>
#include <string>

#include "strix_stream/ss.h"

namespace tsb {

class Error : public std::runtime_error {
 public:
  Error(ss_status s, const std::string& msg) : std::runtime_error(msg), status_(s) {}
  ss_status status() const { return status_; }

 private:
  ss_status status_;
};

[[noreturn]] inline void fail(ss_status s, const std::string& msg) { throw Error(s, msg); }
inline void require(bool ok, ss_status s, const std::string& msg) {
  if (!ok) fail(s, msg);
}

}  // namespace tsb
