// XXH64 on the host, written from the published XXH64 specification (seed 0 unless given; little-endian lanes).
// The descriptor carries the xxh64 of each unit's bytes; the device kernel (kernels.cu) computes the same function.
#pragma once

#include <cstddef>
#include <cstdint>

namespace tsb {

struct Xxh64Consts {
  static constexpr uint64_t k1 = 0x9E3779B185EBCA87ULL;
  static constexpr uint64_t k2 = 0xC2B2AE3D27D4EB4FULL;
  static constexpr uint64_t k3 = 0x165667B19E3779F9ULL;
  static constexpr uint64_t k4 = 0x85EBCA77C2B2AE63ULL;
  static constexpr uint64_t k5 = 0x27D4EB2F165667C5ULL;
};

// Streaming state: feed bytes in any pieces, digest at the end.
class Xxh64State {
 public:
  explicit Xxh64State(uint64_t seed = 0);
  void feed(const void* data, size_t len);
  uint64_t digest() const;

 private:
  uint64_t acc_[4];
  uint64_t seed_;
  uint64_t total_ = 0;
  unsigned char pend_[32];
  size_t npend_ = 0;
};

uint64_t xxh64(const void* data, size_t len, uint64_t seed = 0);

}  // namespace tsb
