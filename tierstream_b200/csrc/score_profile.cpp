#include "score_profile.hpp"

#include <cstring>

#include "errors.hpp"

namespace tsb {

namespace {

// ---- SHA-256 (FIPS 180-4, section 6.2) ----
constexpr uint32_t kK[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5, 0xd807aa98,
    0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786,
    0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8,
    0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13,
    0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819,
    0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a,
    0x5b9cca4f, 0x682e6ff3, 0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
inline uint32_t sigma0(uint32_t x) { return rotr(x, 7) ^ rotr(x, 18) ^ (x >> 3); }
inline uint32_t sigma1(uint32_t x) { return rotr(x, 17) ^ rotr(x, 19) ^ (x >> 10); }
inline uint32_t Sigma0(uint32_t x) { return rotr(x, 2) ^ rotr(x, 13) ^ rotr(x, 22); }
inline uint32_t Sigma1(uint32_t x) { return rotr(x, 6) ^ rotr(x, 11) ^ rotr(x, 25); }
inline uint32_t choose(uint32_t x, uint32_t y, uint32_t z) { return z ^ (x & (y ^ z)); }
inline uint32_t majority(uint32_t x, uint32_t y, uint32_t z) { return (x & y) | (z & (x | y)); }

// One 64-byte block into the state. The eight working variables live in a ring: in round t, variable i (a = 0 ..
// h = 7) is v[(i - t) & 7], so a round writes only the two that change - d's register gains T1 (it is the next
// round's e) and h's register takes T1 + T2 (the next round's a) - and nothing is shifted.
void compress(uint32_t state[8], const unsigned char* block) {
  uint32_t w[64];
  for (int t = 0; t < 16; ++t) {
    w[t] = 0;
    for (int k = 0; k < 4; ++k) w[t] = (w[t] << 8) | block[4 * t + k];  // big-endian words
  }
  for (int t = 16; t < 64; ++t) w[t] = sigma1(w[t - 2]) + w[t - 7] + sigma0(w[t - 15]) + w[t - 16];
  uint32_t v[8];
  std::memcpy(v, state, sizeof v);
  for (int t = 0; t < 64; ++t) {
    auto var = [&](int i) -> uint32_t& { return v[(i - t) & 7]; };
    const uint32_t t1 = var(7) + Sigma1(var(4)) + choose(var(4), var(5), var(6)) + kK[t] + w[t];
    const uint32_t t2 = Sigma0(var(0)) + majority(var(0), var(1), var(2));
    var(3) += t1;
    var(7) = t1 + t2;
  }
  for (int i = 0; i < 8; ++i) state[i] += v[i];  // (after 64 rounds the ring is back at offset 0)
}

void put32(std::string& b, uint32_t v) {
  for (int i = 0; i < 4; ++i) b.push_back(char(v >> (8 * i) & 0xff));
}
void put64(std::string& b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b.push_back(char(v >> (8 * i) & 0xff));
}
uint32_t get32(const unsigned char* p) {
  return uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
}
[[noreturn]] void bad(const std::string& why) { fail(SS_E_INVALID, "dg_score_profile (TSSCPRF1): " + why); }

}  // namespace

std::string sha256(const void* data, size_t len) {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a, 0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  const auto* p = static_cast<const unsigned char*>(data);
  size_t left = len;
  for (; left >= 64; p += 64, left -= 64) compress(h, p);
  unsigned char tail[128] = {};
  std::memcpy(tail, p, left);
  tail[left] = 0x80;
  const size_t blocks = left + 1 + 8 <= 64 ? 1 : 2;
  const uint64_t bits = uint64_t(len) * 8;
  for (int i = 0; i < 8; ++i) tail[blocks * 64 - 1 - i] = (unsigned char)(bits >> (8 * i));
  for (size_t b = 0; b < blocks; ++b) compress(h, tail + 64 * b);
  std::string out(32, '\0');
  for (int i = 0; i < 8; ++i)
    for (int j = 0; j < 4; ++j) out[size_t(4 * i + j)] = char(h[i] >> (24 - 8 * j) & 0xff);
  return out;
}

std::string score_identity(const Desc& d, const std::vector<int>& gated) {
  std::string b;
  put32(b, uint32_t(gated.size()));
  for (size_t g = 0; g < gated.size(); ++g) {
    const Layer& l = d.layers[size_t(gated[g])];
    require(l.hash.size() == size_t(l.n_units), SS_E_INVALID,
            "dg_score_profile: gated layer " + std::to_string(g) +
                " has no per-unit hashes in the descriptor (a profile is bound to them)");
    put32(b, uint32_t(l.index));
    put32(b, uint32_t(l.n_units));
    put64(b, l.unit_bytes);
    for (uint64_t h : l.hash) put64(b, h);
  }
  return sha256(b.data(), b.size());
}

// TSSCPRF1: magic[8], u32 version (1), u32 n_gated, u32 units per gated layer, identity[32], u32 prov_len,
// prov[prov_len], per gated layer units^2 u32 counts, sha256[32] of everything before it. Checked front to back,
// each field against this context before the next is read.
ScoreProfile check_score_profile(const void* data, uint64_t len, const std::vector<uint32_t>& units,
                                 const std::string& identity) {
  if (!data) bad("null data");
  const auto* bytes = static_cast<const unsigned char*>(data);
  const uint64_t n_gated = units.size();
  const uint64_t head = 8 + 4 + 4 + 4 * n_gated + 32 + 4;  // through prov_len
  if (len < head) bad("truncated header (" + std::to_string(len) + " bytes)");
  uint64_t at = 0;
  auto word = [&] {
    const uint32_t v = get32(bytes + at);
    at += 4;
    return v;
  };
  if (std::memcmp(bytes, "TSSCPRF1", 8) != 0) bad("bad magic");
  at = 8;
  if (const uint32_t version = word(); version != 1) bad("unsupported version " + std::to_string(version));
  if (const uint32_t n = word(); n != n_gated)
    bad("n_gated " + std::to_string(n) + " != the context's " + std::to_string(n_gated));
  for (size_t g = 0; g < units.size(); ++g)
    if (const uint32_t u = word(); u != units[g])
      bad("units of gated layer " + std::to_string(g) + " are " + std::to_string(u) + ", the context has " +
          std::to_string(units[g]));
  const unsigned char* id = bytes + at;
  at += 32;
  const uint32_t prov = word();
  if (prov > 4096) bad("provenance longer than 4096 bytes");
  uint64_t cells = 0;
  for (uint32_t u : units) cells += uint64_t(u) * u;  // (units <= 65536 per layer: checked by the open)
  const uint64_t want = head + prov + 4 * cells + 32;
  if (len != want) bad("size " + std::to_string(len) + " != " + std::to_string(want) + " (header + cells + checksum)");
  if (identity.size() != 32 || std::memcmp(id, identity.data(), 32) != 0)
    bad("identity mismatch (another model, layer set or descriptor)");
  if (sha256(bytes, size_t(len - 32)) != std::string(reinterpret_cast<const char*>(bytes + len - 32), 32))
    bad("checksum mismatch");
  ScoreProfile out;
  out.provenance.assign(reinterpret_cast<const char*>(bytes + at), prov);
  at += prov;
  out.cells.reserve(units.size());
  for (uint32_t u : units) {
    std::vector<uint32_t> layer(size_t(u) * u);
    for (uint32_t& v : layer) v = word();
    out.cells.push_back(std::move(layer));
  }
  return out;
}

}  // namespace tsb
