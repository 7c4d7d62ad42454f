/* CPU restatement of the reference's hot-path arithmetic. TEST INFRASTRUCTURE ONLY (see oracle.h). */
#include "oracle.h"

#include <string.h>

#define P1 0x9E3779B185EBCA87ULL
#define P2 0xC2B2AE3D27D4EB4FULL
#define P3 0x165667B19E3779F9ULL
#define P4 0x85EBCA77C2B2AE63ULL
#define P5 0x27D4EB2F165667C5ULL

static uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
static uint64_t rd64(const uint8_t* p) {
  uint64_t v = 0;
  for (int k = 7; k >= 0; --k) v = (v << 8) | p[k];
  return v;
}
static uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
static uint64_t xround(uint64_t acc, uint64_t w) { return rotl(acc + w * P2, 31) * P1; }

typedef struct {
  uint64_t v[4], seed, total;
  uint8_t buf[32];
  size_t n;
} xstate;

static void xinit(xstate* s, uint64_t seed) {
  s->v[0] = seed + P1 + P2;
  s->v[1] = seed + P2;
  s->v[2] = seed;
  s->v[3] = seed - P1;
  s->seed = seed;
  s->total = 0;
  s->n = 0;
}

/* xxh64.cpp:50-75 (Xxh64::update) */
static void xfeed(xstate* s, const uint8_t* p, size_t len) {
  s->total += len;
  while (len) {
    size_t take = 32 - s->n < len ? 32 - s->n : len;
    memcpy(s->buf + s->n, p, take);
    s->n += take;
    p += take;
    len -= take;
    if (s->n == 32) {
      for (int k = 0; k < 4; ++k) s->v[k] = xround(s->v[k], rd64(s->buf + 8 * k));
      s->n = 0;
    }
  }
}

/* the final mix: xor-shifts by 33, 29 and 32 with multiplies by P2 and P3 between them */
static uint64_t xavalanche(uint64_t h) {
  h = (h ^ (h >> 33)) * P2;
  h = (h ^ (h >> 29)) * P3;
  return h ^ (h >> 32);
}

/* xxh64.cpp:77-106 (Xxh64::digest) */
static uint64_t xdigest(const xstate* s) {
  uint64_t h;
  if (s->total >= 32) {
    h = rotl(s->v[0], 1) + rotl(s->v[1], 7) + rotl(s->v[2], 12) + rotl(s->v[3], 18);
    for (int k = 0; k < 4; ++k) h = (h ^ xround(0, s->v[k])) * P1 + P4;
  } else {
    h = s->seed + P5;
  }
  h += s->total;
  /* the buffered tail: 8-byte lanes, then one 4-byte word, then single bytes */
  size_t at = 0;
  for (; at + 8 <= s->n; at += 8) h = rotl(h ^ xround(0, rd64(s->buf + at)), 27) * P1 + P4;
  if (at + 4 <= s->n) {
    h = rotl(h ^ (uint64_t)rd32(s->buf + at) * P1, 23) * P2 + P3;
    at += 4;
  }
  for (; at < s->n; ++at) h = rotl(h ^ (uint64_t)s->buf[at] * P5, 11) * P1;
  return xavalanche(h);
}

uint64_t orc_xxh64(const void* data, size_t len, uint64_t seed) {
  xstate s;
  xinit(&s, seed);
  xfeed(&s, (const uint8_t*)data, len);
  return xdigest(&s);
}

uint64_t orc_xxh64_spans(const void* const* ptrs, const uint64_t* lens, uint32_t n, uint64_t seed) {
  xstate s;
  xinit(&s, seed);
  for (uint32_t i = 0; i < n; ++i) xfeed(&s, (const uint8_t*)ptrs[i], (size_t)lens[i]);
  return xdigest(&s);
}

/* tests/fixture.hpp:16-22 (byte_at) */
void orc_fill_bytes(uint64_t file_id, uint64_t first, uint64_t n, uint8_t* out) {
  for (uint64_t j = 0; j < n; ++j) {
    const uint64_t i = first + j;
    uint64_t x = (i + 1) * 0x9E3779B97F4A7C15ULL ^ (file_id + 7) * 0xC2B2AE3D27D4EB4FULL;
    x ^= x >> 29;
    x *= 0xBF58476D1CE4E5B9ULL;
    x ^= x >> 32;
    out[j] = (uint8_t)x;
  }
}

/* tests/test_dg_cuda.cu:103-114 (the per-unit checksum through the slot table) */
uint64_t orc_checksum(const uint8_t* p, uint64_t n) {
  uint64_t s = 0;
  for (uint64_t i = 0; i < n; ++i) s += (uint64_t)p[i] * (i % 251 + 1);
  return s;
}

/* dg_kernels.cu:49-87 (export_kernel's mask and bad-id rule) */
uint64_t orc_export_mask(const int32_t* slot_of, uint32_t base, uint32_t units, const int32_t* ids, uint32_t n,
                         uint32_t* bad) {
  uint64_t mask = 0;
  *bad = 0;
  for (uint32_t t = 0; t < n && t < 64; ++t) {
    const uint32_t id = (uint32_t)ids[t];
    if (id >= units) *bad = 1;
    else if (slot_of[base + id] < 0) mask |= 1ULL << t;
  }
  return mask;
}

/* ss.h:952-962 (ss_dg_slot) */
int32_t orc_dg_slot(const int32_t* slot_of, const uint32_t* unit_base, uint32_t g, int32_t id, uint32_t guard,
                    uint32_t abort_flag, uint32_t* absent_err) {
  if (abort_flag) return (int32_t)guard;
  const uint32_t b = unit_base[g];
  if ((uint32_t)id >= unit_base[g + 1] - b) return (int32_t)guard;
  const int32_t s = slot_of[b + (uint32_t)id];
  if (s >= 0) return s;
  if (absent_err) *absent_err |= 1u;
  return (int32_t)guard;
}
