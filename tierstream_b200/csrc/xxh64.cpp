#include "xxh64.hpp"

#include <cstring>

namespace tsb {
namespace {

using K = Xxh64Consts;

inline uint64_t rotl64(uint64_t v, unsigned r) { return (v << r) | (v >> (64 - r)); }

inline uint64_t load_le64(const unsigned char* p) {
  return uint64_t(p[0]) | uint64_t(p[1]) << 8 | uint64_t(p[2]) << 16 | uint64_t(p[3]) << 24 | uint64_t(p[4]) << 32 |
         uint64_t(p[5]) << 40 | uint64_t(p[6]) << 48 | uint64_t(p[7]) << 56;
}

inline uint32_t load_le32(const unsigned char* p) {
  return uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
}

// One lane step of the stripe loop.
inline uint64_t lane_step(uint64_t acc, uint64_t word) { return rotl64(acc + word * K::k2, 31) * K::k1; }

inline uint64_t fold_lane(uint64_t h, uint64_t lane) { return (h ^ lane_step(0, lane)) * K::k1 + K::k4; }

}  // namespace

Xxh64State::Xxh64State(uint64_t seed) : seed_(seed) {
  acc_[0] = seed + K::k1 + K::k2;
  acc_[1] = seed + K::k2;
  acc_[2] = seed;
  acc_[3] = seed - K::k1;
}

void Xxh64State::feed(const void* data, size_t len) {
  const unsigned char* p = static_cast<const unsigned char*>(data);
  total_ += len;
  if (npend_) {  // complete a buffered stripe first
    const size_t take = len < 32 - npend_ ? len : 32 - npend_;
    std::memcpy(pend_ + npend_, p, take);
    npend_ += take;
    p += take;
    len -= take;
    if (npend_ < 32) return;
    for (int l = 0; l < 4; ++l) acc_[l] = lane_step(acc_[l], load_le64(pend_ + 8 * l));
    npend_ = 0;
  }
  for (; len >= 32; p += 32, len -= 32)
    for (int l = 0; l < 4; ++l) acc_[l] = lane_step(acc_[l], load_le64(p + 8 * l));
  std::memcpy(pend_, p, len);
  npend_ = len;
}

uint64_t Xxh64State::digest() const {
  uint64_t h;
  if (total_ >= 32) {
    h = rotl64(acc_[0], 1) + rotl64(acc_[1], 7) + rotl64(acc_[2], 12) + rotl64(acc_[3], 18);
    for (int l = 0; l < 4; ++l) h = fold_lane(h, acc_[l]);
  } else {
    h = seed_ + K::k5;
  }
  h += total_;
  size_t off = 0;
  for (; off + 8 <= npend_; off += 8) h = rotl64(h ^ lane_step(0, load_le64(pend_ + off)), 27) * K::k1 + K::k4;
  if (off + 4 <= npend_) {
    h = rotl64(h ^ (uint64_t(load_le32(pend_ + off)) * K::k1), 23) * K::k2 + K::k3;
    off += 4;
  }
  for (; off < npend_; ++off) h = rotl64(h ^ (uint64_t(pend_[off]) * K::k5), 11) * K::k1;
  h ^= h >> 33;
  h *= K::k2;
  h ^= h >> 29;
  h *= K::k3;
  h ^= h >> 32;
  return h;
}

uint64_t xxh64(const void* data, size_t len, uint64_t seed) {
  Xxh64State s(seed);
  s.feed(data, len);
  return s.digest();
}

}  // namespace tsb
