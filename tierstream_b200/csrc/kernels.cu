// Device kernels of the B200 runtime (sm_100a). Byte movement and control only: no tensor-core work exists on this
// path. See kernels.hpp for the launch contracts.
#include <atomic>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.hpp"

namespace tsb {
namespace dev {
namespace {

// ---------------------------------------------------------------------------------------------------------------
// K1 / K5: the batched copy ("land") kernel.
// The copies are cut into 64 KiB chunks; block i takes chunks i, i + grid, ... Each chunk moves 16-byte vectors with
// eight loads in flight per thread (mapped pinned host memory is read over PCIe, HBM or a peer over NVLink). The last
// block to finish publishes the batch's entries and ready word, so one launch replaces a copy per part plus a stream
// write per entry.
// ---------------------------------------------------------------------------------------------------------------
constexpr uint32_t kChunk = 64u << 10;
constexpr int kCopyThreads = 512;

__device__ __forceinline__ void copy_vec(const uint4* __restrict__ s, uint4* __restrict__ d, uint32_t n16) {
  uint32_t i = threadIdx.x;
  constexpr uint32_t U = 8;
  for (; i + (U - 1) * kCopyThreads < n16; i += U * kCopyThreads) {
    uint4 v[U];
#pragma unroll
    for (uint32_t u = 0; u < U; ++u) v[u] = __ldcs(s + i + u * kCopyThreads);
#pragma unroll
    for (uint32_t u = 0; u < U; ++u) d[i + u * kCopyThreads] = v[u];
  }
  for (; i < n16; i += kCopyThreads) d[i] = __ldcs(s + i);
}

// Any alignment: bytes up to the next 16-byte boundary of both sides (when they share it), vectors, then bytes.
__device__ void copy_range(const uint8_t* s, uint8_t* d, uint64_t n) {
  if (((reinterpret_cast<uintptr_t>(s) ^ reinterpret_cast<uintptr_t>(d)) & 15u) == 0) {
    const uint32_t head = uint32_t((16u - (reinterpret_cast<uintptr_t>(s) & 15u)) & 15u);
    const uint32_t h = head < n ? head : uint32_t(n);
    if (threadIdx.x < h) d[threadIdx.x] = s[threadIdx.x];
    const uint64_t body = (n - h) / 16;
    copy_vec(reinterpret_cast<const uint4*>(s + h), reinterpret_cast<uint4*>(d + h), uint32_t(body));
    const uint64_t done = h + body * 16;
    if (threadIdx.x < n - done) d[done + threadIdx.x] = s[done + threadIdx.x];
    return;
  }
  for (uint64_t i = threadIdx.x; i < n; i += kCopyThreads) d[i] = s[i];
}

__global__ __launch_bounds__(kCopyThreads) void batch_kernel(const __grid_constant__ Batch b) {
  __shared__ uint32_t first_chunk[kMaxCopies + 1];
  __shared__ uint32_t is_last;
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (uint32_t c = 0; c < b.n_copies; ++c) {
      first_chunk[c] = acc;
      acc += uint32_t((b.copies[c].bytes + kChunk - 1) / kChunk);
    }
    first_chunk[b.n_copies] = acc;
  }
  __syncthreads();
  const uint32_t total = first_chunk[b.n_copies];
  uint32_t c = 0;
  for (uint32_t k = blockIdx.x; k < total; k += gridDim.x) {
    while (c + 1 < b.n_copies && first_chunk[c + 1] <= k) ++c;  // k only grows: the copy index only grows
    const Copy& cp = b.copies[c];
    const uint64_t off = uint64_t(k - first_chunk[c]) * kChunk;
    const uint64_t n = cp.bytes - off < kChunk ? cp.bytes - off : kChunk;
    const uint8_t* s = static_cast<const uint8_t*>(cp.src) + off;
    uint8_t* d = static_cast<uint8_t*>(cp.dst) + off;
    if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d) | n) & 15u) == 0)
      copy_vec(reinterpret_cast<const uint4*>(s), reinterpret_cast<uint4*>(d), uint32_t(n / 16));
    else
      copy_range(s, d, n);
  }
  if (!b.done_counter) return;
  // the last block publishes: every block's stores are fenced before its arrival
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) is_last = atomicAdd(b.done_counter, 1u) == gridDim.x - 1 ? 1u : 0u;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (uint32_t e = threadIdx.x; e < b.n_entries; e += kCopyThreads)
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(b.slot_of + b.entry_key[e]), "r"(b.entry_val[e])
                 : "memory");
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    *b.done_counter = 0;
    if (b.ready_word) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(b.ready_word), "r"(b.ready_val) : "memory");
  }
}

// ---------------------------------------------------------------------------------------------------------------
// K3: xxh64 of whole units. XXH64 is four serial lane chains per unit (a 64-bit add, rotate and multiply per 32-byte
// stripe and lane), so one unit's rate is set by the latency of that chain; the kernel keeps each chain as short as
// the arithmetic allows and runs many units at once. A CTA is two independent warps; a warp serves 8 units, thread t
// carrying accumulator t & 3 of unit t >> 2. The input product x * P2 of eight stripes is computed ahead of their
// steps, so the chain itself is an add with carry, two funnel shifts and one widening multiply with its two cross
// products. Bytes are staged in shared memory by TMA bulk copies (one cp.async.bulk per unit, chunk and span, issued
// by the unit's own lane, completing on the warp's mbarrier of that stage) through a ring of 4 x 2 KiB stages per
// unit; unit rings are offset by 32 B in rotation so a half-warp's 32-byte reads of four units fall in distinct banks.
// Units whose spans are not 16-byte aligned, or not 32-byte multiples except the last, take a one-lane path from
// global memory. Every mbarrier wait is bounded (2 s of globaltimer, or an iteration cap); one that runs out is
// counted in the launch's timeout word, reports the warp's units as failed (hash 0) and returns after a bounded wait
// for the copies already issued.
// ---------------------------------------------------------------------------------------------------------------
constexpr uint64_t X1 = 0x9E3779B185EBCA87ULL, X2 = 0xC2B2AE3D27D4EB4FULL, X3 = 0x165667B19E3779F9ULL,
                   X4 = 0x85EBCA77C2B2AE63ULL, X5 = 0x27D4EB2F165667C5ULL;
constexpr uint32_t kX1lo = uint32_t(X1), kX1hi = uint32_t(X1 >> 32);
constexpr int kHashWarpUnits = 8, kHashWarps = 2, kHashUnits = kHashWarpUnits * kHashWarps;
constexpr int kHashStages = 4, kHashChunk = 2048;
constexpr int kHashRegion = kHashStages * kHashChunk + 128;  // one unit's ring, plus room for the bank offset
constexpr size_t kHashWarpBytes = size_t(kHashWarpUnits) * kHashRegion;
constexpr size_t kHashSmem = size_t(kHashWarps) * kHashWarpBytes + size_t(kHashWarps) * kHashStages * 8;
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ uint32_t g_xxh64_timeouts;

__device__ __forceinline__ uint64_t rotl64(uint64_t v, uint32_t r) { return (v << r) | (v >> (64 - r)); }
__device__ __forceinline__ uint64_t lane_step(uint64_t acc, uint64_t w) { return rotl64(acc + w * X2, 31) * X1; }

// One stripe step of a lane chain, acc = rotl(acc + y, 31) * P1 with y = x * P2 already computed: the add with carry,
// the rotation as two funnel shifts ({hi:lo} << 31 | {hi:lo} >> 33), the product mod 2^64 as lo x P1lo widened plus
// the two cross products into the high word.
__device__ __forceinline__ void chain_step(uint32_t& lo, uint32_t& hi, uint64_t y) {
  uint32_t rl, rh;
  asm("{\n\t.reg .u32 tl, th;\n\t"
      "add.cc.u32 tl, %2, %4;\n\t"
      "addc.u32 th, %3, %5;\n\t"
      "shf.l.wrap.b32 %0, th, tl, 31;\n\t"
      "shf.l.wrap.b32 %1, tl, th, 31;\n\t"
      "}"
      : "=r"(rl), "=r"(rh)
      : "r"(lo), "r"(hi), "r"(uint32_t(y)), "r"(uint32_t(y >> 32)));
  const uint64_t d = uint64_t(rl) * kX1lo;
  lo = uint32_t(d);
  hi = uint32_t(d >> 32) + rl * kX1hi + rh * kX1lo;
}
// n (1..64) stripes of this thread's lane (its word every 32 bytes from w) into acc; the input products eight ahead.
__device__ __forceinline__ uint64_t chain_stripes(uint64_t acc, const uint64_t* w, uint32_t n) {
  uint32_t lo = uint32_t(acc), hi = uint32_t(acc >> 32);
  if (n == kHashChunk / 32) {
#pragma unroll 2
    for (int g = 0; g < kHashChunk / 32; g += 8) {
      uint64_t y[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) y[k] = w[4 * (g + k)] * X2;
#pragma unroll
      for (int k = 0; k < 8; ++k) chain_step(lo, hi, y[k]);
    }
  } else {
    for (uint32_t s = 0; s < n; ++s) chain_step(lo, hi, w[4 * s] * X2);
  }
  return uint64_t(hi) << 32 | lo;
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded: true when the phase completed, false after kWaitNs or the iteration cap.
__device__ bool mbar_wait(uint64_t* b, uint32_t parity) {
  if (mbar_try_wait(b, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63u) == 0 && globaltimer_ns() - t0 > kWaitNs) return false;
  }
  return false;
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// The byte at stream position p of a unit (spans back to back).
__device__ __forceinline__ uint8_t unit_byte(const HashUnit& u, uint64_t p) {
  for (uint32_t s = 0; s < u.n_spans; ++s) {
    if (p < u.bytes[s]) return u.span[s][p];
    p -= u.bytes[s];
  }
  return 0;
}
__device__ __forceinline__ uint64_t unit_le64(const HashUnit& u, uint64_t p) {
  uint64_t v = 0;
  for (int k = 7; k >= 0; --k) v = (v << 8) | unit_byte(u, p + uint64_t(k));
  return v;
}

// Everything after the stripes: the merge of the lanes (when total >= 32), the tail, the avalanche.
__device__ uint64_t finish_hash(const HashUnit& u, const uint64_t v[4], uint64_t total, uint64_t body) {
  uint64_t h;
  if (total >= 32) {
    h = rotl64(v[0], 1) + rotl64(v[1], 7) + rotl64(v[2], 12) + rotl64(v[3], 18);
    for (int l = 0; l < 4; ++l) h = (h ^ lane_step(0, v[l])) * X1 + X4;
  } else {
    h = X5;
  }
  h += total;
  uint64_t p = body;
  for (; p + 8 <= total; p += 8) h = rotl64(h ^ lane_step(0, unit_le64(u, p)), 27) * X1 + X4;
  if (p + 4 <= total) {
    const uint32_t w = uint32_t(unit_byte(u, p)) | uint32_t(unit_byte(u, p + 1)) << 8 |
                       uint32_t(unit_byte(u, p + 2)) << 16 | uint32_t(unit_byte(u, p + 3)) << 24;
    h = rotl64(h ^ (uint64_t(w) * X1), 23) * X2 + X3;
    p += 4;
  }
  for (; p < total; ++p) h = rotl64(h ^ (uint64_t(unit_byte(u, p)) * X5), 11) * X1;
  h ^= h >> 33;
  h *= X2;
  h ^= h >> 29;
  h *= X3;
  h ^= h >> 32;
  return h;
}

__device__ __forceinline__ uint64_t seed_acc(uint32_t l) {  // seed 0
  return l == 0 ? X1 + X2 : l == 1 ? X2 : l == 2 ? 0 : uint64_t(0) - X1;
}

// Where a launch's units come from and where their hashes go. A table in device memory (tsb_xxh64_units and the
// open's checks): out[i] = the hash; with expectations, a mismatch (or a failed unit) sets bad[i] and adds 1 to
// *mismatches.
struct TableUnits {
  const HashUnit* units;
  const uint64_t* expect;
  uint64_t* out;
  uint32_t* bad;
  uint32_t* mismatches;
  __device__ HashUnit unit(uint32_t i) const { return units[i]; }
  __device__ void result(uint32_t i, uint64_t h, bool failed) const {
    out[i] = h;
    if (failed || (expect && expect[i] != h)) {
      if (bad) bad[i] = 1;
      if (expect && mismatches) atomicAdd(mismatches, 1u);
    }
  }
};
// Landed slots of a device-gated arena, by value in the launch: unit i is key[i] in slot[i]; compared with
// expect[key]. A mismatch adds 1 to *bad_count and, while the log has room, writes (key, slot) to the mapped log.
struct LandedUnits {
  const VerifyBatch* b;
  __device__ HashUnit unit(uint32_t i) const {
    HashUnit u{};
    u.n_spans = b->n_parts;
    const uint64_t slot = uint64_t(uint32_t(b->slot[i]));
    for (uint32_t p = 0; p < b->n_parts && p < 4; ++p) {
      u.span[p] = b->arena[p] + slot * b->part_bytes[p];
      u.bytes[p] = b->part_bytes[p];
    }
    return u;
  }
  __device__ void result(uint32_t i, uint64_t h, bool failed) const {
    if (!failed && b->expect[b->key[i]] == h) return;
    const uint32_t at = atomicAdd(b->bad_count, 1u);
    if (at < kBadLog) {
      volatile uint32_t* log = b->bad_log;
      log[2 * at] = b->key[i];
      log[2 * at + 1] = uint32_t(b->slot[i]);
    }
    __threadfence_system();  // the entry before the flag
    *reinterpret_cast<volatile uint32_t*>(b->bad_flag) = 1u;
    __threadfence_system();
  }
};

// One warp's 8 units (first .. first + 7) through its region of shared memory and its stage barriers.
template <class Src>
__device__ void hash_warp(const Src& src, uint32_t n, uint32_t first, uint8_t* wsmem, uint64_t* bars,
                          uint32_t* timeouts) {
  const uint32_t lane = threadIdx.x & 31u, q = lane >> 2, l = lane & 3u;
  // lane i < 8 holds unit first + i: its spans, whether it takes the staged path, its staged (stripe) bytes
  HashUnit mine{};
  uint64_t body = 0;
  if (lane < uint32_t(kHashWarpUnits) && first + lane < n) {
    mine = src.unit(first + lane);
    bool ok = mine.n_spans >= 1 && mine.n_spans <= 4;
    uint64_t total = 0;
#pragma unroll
    for (uint32_t s = 0; s < 4; ++s) {
      if (s >= mine.n_spans) break;
      ok = ok && (reinterpret_cast<uintptr_t>(mine.span[s]) & 15u) == 0 &&
           (s + 1 == mine.n_spans || mine.bytes[s] % 32 == 0);
      total += mine.bytes[s];
    }
    body = ok ? total / 32 * 32 : 0;
  }
  const uint32_t nchunks = __reduce_max_sync(0xffffffffu, uint32_t((body + kHashChunk - 1) / kHashChunk));
  const uint64_t body_q = __shfl_sync(0xffffffffu, body, int(q));
  uint8_t* region = wsmem + size_t(lane) * kHashRegion + (lane & 3u) * 32;  // valid for lane < 8
  const uint8_t* rd = wsmem + size_t(q) * kHashRegion + (q & 3u) * 32 + 8 * l;
  if (lane == 0 && nchunks) {
    for (int s = 0; s < kHashStages; ++s) mbar_init(bars + s, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  // chunk c of every unit into stage c % kHashStages: lane 0 arms the stage's barrier with the chunk's bytes, each
  // unit's lane issues its copies (one per span the chunk touches)
  auto issue = [&](uint32_t c) {
    uint64_t* bar = bars + (c % kHashStages);
    const uint64_t start = uint64_t(c) * kHashChunk;
    const uint32_t bytes = start < body ? uint32_t(body - start < kHashChunk ? body - start : kHashChunk) : 0u;
    const uint32_t all = __reduce_add_sync(0xffffffffu, bytes);
    if (lane == 0) mbar_arrive_expect_tx(bar, all);
    __syncwarp();
    if (!bytes) return;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the stage was last read by ordinary loads
    uint8_t* dst = region + size_t(c % kHashStages) * kHashChunk;
    uint64_t p = start;
    uint32_t left = bytes;
#pragma unroll
    for (uint32_t s = 0; s < 4; ++s) {
      if (s >= mine.n_spans || !left) break;
      if (p >= mine.bytes[s]) {
        p -= mine.bytes[s];
        continue;
      }
      const uint64_t avail = mine.bytes[s] - p;
      const uint32_t take = avail < left ? uint32_t(avail) : left;
      bulk_load(dst, mine.span[s] + p, take, bar);
      dst += take;
      left -= take;
      p = 0;
    }
  };
  for (uint32_t c = 0; c < uint32_t(kHashStages) && c < nchunks; ++c) issue(c);
  uint64_t acc = seed_acc(l);
  bool timed_out = false;
  uint32_t c = 0;
  for (; c < nchunks; ++c) {
    const bool ok = mbar_wait(bars + (c % kHashStages), (c / kHashStages) & 1u);
    if (!__all_sync(0xffffffffu, ok)) {
      timed_out = true;
      break;
    }
    const uint64_t* w = reinterpret_cast<const uint64_t*>(rd + size_t(c % kHashStages) * kHashChunk);
    const uint64_t start = uint64_t(c) * kHashChunk;
    const uint32_t nq = start < body_q ? uint32_t((body_q - start < kHashChunk ? body_q - start : kHashChunk) / 32) : 0u;
    if (nq) acc = chain_stripes(acc, w, nq);
    __syncwarp();  // every lane is done with the stage before it is refilled
    if (c + kHashStages < nchunks) issue(c + kHashStages);
  }
  if (timed_out) {
    if (lane == 0) atomicAdd(timeouts ? timeouts : &g_xxh64_timeouts, 1u);
    // the copies already issued (stages c .. c + kHashStages - 1) land before the warp leaves, each wait bounded
    for (uint32_t k = c; k < nchunks && k < c + kHashStages; ++k)
      (void)mbar_wait(bars + (k % kHashStages), (k / kHashStages) & 1u);
    if (lane < uint32_t(kHashWarpUnits) && first + lane < n) src.result(first + lane, 0, true);
    return;
  }
  // each quad's accumulators on its lane 0, which finishes unit first + q
  uint64_t v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = __shfl_sync(0xffffffffu, acc, int((lane & ~3u) + k));
  const uint32_t idx = first + q;
  if (l != 0 || idx >= n) return;
  const HashUnit u = src.unit(idx);
  uint64_t t = 0;
  for (uint32_t s = 0; s < u.n_spans && s < 4; ++s) t += u.bytes[s];
  uint64_t h;
  if (body_q) {
    h = finish_hash(u, v, t, body_q);
  } else {  // shorter than a stripe, or the one-lane path from global memory
    uint64_t a[4] = {seed_acc(0), seed_acc(1), seed_acc(2), seed_acc(3)};
    const uint64_t bb = t / 32 * 32;
    for (uint64_t p = 0; p < bb; p += 32)
      for (int k = 0; k < 4; ++k) a[k] = lane_step(a[k], unit_le64(u, p + 8 * uint64_t(k)));
    h = finish_hash(u, a, t, bb);
  }
  src.result(idx, h, false);
}

__global__ __launch_bounds__(32 * kHashWarps) void xxh64_kernel(const HashUnit* __restrict__ units, uint32_t n,
                                                                const uint64_t* __restrict__ expect,
                                                                uint64_t* __restrict__ out, uint32_t* __restrict__ bad,
                                                                uint32_t* __restrict__ mismatches, uint32_t* timeouts) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t w = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kHashWarps * kHashWarpBytes) + w * kHashStages;
  const TableUnits src{units, expect, out, bad, mismatches};
  hash_warp(src, n, (blockIdx.x * kHashWarps + w) * kHashWarpUnits, smem + w * kHashWarpBytes, bars, timeouts);
}

__global__ __launch_bounds__(32 * kHashWarps) void xxh64_landed_kernel(const __grid_constant__ VerifyBatch b) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t w = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kHashWarps * kHashWarpBytes) + w * kHashStages;
  const LandedUnits src{&b};
  hash_warp(src, b.n, (blockIdx.x * kHashWarps + w) * kHashWarpUnits, smem + w * kHashWarpBytes, bars, b.timeouts);
  __syncthreads();
  if (threadIdx.x != 0) return;
  __threadfence_system();  // this CTA's log entries before the launch's done word
  if (atomicAdd(b.done_cnt, 1u) != gridDim.x - 1) return;
  *reinterpret_cast<volatile uint32_t*>(b.done_cnt) = 0u;
  __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(b.done_word), "r"(b.done_val) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// K4: HBM -> HBM moves staged through shared memory by TMA bulk copies (reset compaction). One warp per CTA, its lane 0
// issuing: every 64 KiB chunk is a bulk load global -> shared (completing on the stage's mbarrier) followed by a bulk
// store shared -> global, through a ring of 3 stages, with the loads of the next two chunks in flight while a store
// drains. Copies must be 16-byte aligned with 16-byte multiple sizes (the host checks; the land kernel takes the
// rest). The last CTA publishes entries and the ready word as K1 does. A load wait that runs out (2 s) is counted in
// g_move_timeouts; that CTA waits (bounded) for its loads in flight and for its stores, and leaves without
// publishing, so the batch's publication never happens and the host reports the failure.
// ---------------------------------------------------------------------------------------------------------------
constexpr int kMoveStages = 3;
constexpr uint32_t kMoveChunk = 64u << 10;
constexpr size_t kMoveSmem = size_t(kMoveStages) * kMoveChunk + kMoveStages * 8;

__device__ uint32_t g_move_timeouts;

__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_reads() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ __launch_bounds__(32) void move_kernel(const __grid_constant__ Batch b) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t first_chunk[kMaxCopies + 1];
  if (threadIdx.x != 0) return;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(kMoveStages) * kMoveChunk);
  uint32_t acc = 0;
  for (uint32_t c = 0; c < b.n_copies; ++c) {
    first_chunk[c] = acc;
    acc += uint32_t((b.copies[c].bytes + kMoveChunk - 1) / kMoveChunk);
  }
  first_chunk[b.n_copies] = acc;
  const uint32_t total = acc;
  const uint32_t mine = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0u;
  for (int st = 0; st < kMoveStages; ++st) mbar_init(bars + st, 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  // chunk j of this CTA: global chunk blockIdx.x + j * gridDim.x; the copy index only grows with j
  uint32_t load_c = 0, store_c = 0;
  auto locate = [&](uint32_t j, uint32_t& c, const uint8_t*& src, uint8_t*& dst, uint32_t& n) {
    const uint32_t k = blockIdx.x + j * gridDim.x;
    while (c + 1 < b.n_copies && first_chunk[c + 1] <= k) ++c;
    const uint64_t off = uint64_t(k - first_chunk[c]) * kMoveChunk;
    const uint64_t left = b.copies[c].bytes - off;
    n = uint32_t(left < kMoveChunk ? left : kMoveChunk);
    src = static_cast<const uint8_t*>(b.copies[c].src) + off;
    dst = static_cast<uint8_t*>(b.copies[c].dst) + off;
  };
  auto issue_load = [&](uint32_t j) {
    const uint8_t* src;
    uint8_t* dst;
    uint32_t n;
    locate(j, load_c, src, dst, n);
    uint64_t* bar = bars + (j % kMoveStages);
    mbar_arrive_expect_tx(bar, n);
    bulk_load(smem + size_t(j % kMoveStages) * kMoveChunk, src, n, bar);
  };
  for (uint32_t j = 0; j < uint32_t(kMoveStages) && j < mine; ++j) issue_load(j);
  bool ok = true;
  uint32_t j = 0;
  for (; j < mine; ++j) {
    if (!mbar_wait(bars + (j % kMoveStages), (j / kMoveStages) & 1u)) {
      ok = false;
      break;
    }
    const uint8_t* src;
    uint8_t* dst;
    uint32_t n;
    locate(j, store_c, src, dst, n);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    bulk_store(dst, smem + size_t(j % kMoveStages) * kMoveChunk, n);
    bulk_commit();
    if (j + kMoveStages < mine) {
      bulk_wait_reads();  // the stage is free once the store has read it
      issue_load(j + kMoveStages);
    }
  }
  if (!ok) {
    atomicAdd(&g_move_timeouts, 1u);
    for (uint32_t k = j; k < mine && k < j + kMoveStages; ++k)
      (void)mbar_wait(bars + (k % kMoveStages), (k / kMoveStages) & 1u);
    bulk_wait_all();
    return;
  }
  bulk_wait_all();  // every store of this CTA has landed
  if (!b.done_counter) return;
  asm volatile("fence.proxy.async;" ::: "memory");
  __threadfence();
  if (atomicAdd(b.done_counter, 1u) != gridDim.x - 1) return;
  __threadfence();
  for (uint32_t e = 0; e < b.n_entries; ++e)
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(b.slot_of + b.entry_key[e]), "r"(b.entry_val[e])
                 : "memory");
  __threadfence_system();
  *b.done_counter = 0;
  if (b.ready_word) asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(b.ready_word), "r"(b.ready_val) : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// K2: device-gated decode control. The words they share with the service thread follow the reference's protocol
// (dg_kernels.cu:41-135): begin authorizes one sequence; export writes the record and flag; wait polls the ready
// word; end folds the errors and writes done. Here ready lives in device memory (written by the land kernel or a
// stream write), the export mask is a warp ballot, and every wait is bounded by a globaltimer deadline.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acq_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int32_t ld_acq_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acq_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_vol(uint32_t* p, uint32_t v) { *reinterpret_cast<volatile uint32_t*>(p) = v; }
__device__ __forceinline__ uint32_t ld_vol(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }

// The token's first error keeps its code; abort is sticky.
__device__ void raise(const DgDev& d, uint32_t code, uint32_t aux) {
  if (atomicCAS(d.err_code, 0u, code) == 0u) *d.err_aux = aux;
  if (code == kDgTimeout) atomicAdd(d.err_count, 1u);
  atomicExch(d.abort, 1u);
}

__global__ void dg_begin_kernel(DgDev d) {
  const uint32_t seq = *d.seq + 1u;
  *d.seq = seq;
  if (ld_acq_sys(d.host_seq) != seq) raise(d, kDgDesync, seq);
  __threadfence_system();
  st_vol(d.began, seq);
}

__global__ __launch_bounds__(64) void dg_export_kernel(DgDev d, uint32_t g, const int32_t* ids, uint32_t n,
                                                       uint32_t n_pred) {
  __shared__ uint32_t mask_w[2], bad_w[2];
  const uint32_t t = threadIdx.x, warp = t >> 5;
  const uint32_t seq = *d.seq;
  const uint32_t base = d.unit_base[g], units = d.unit_base[g + 1] - base;
  bool miss = false, bad = false;
  if (t < n) {
    const uint32_t id = uint32_t(ids[t]);
    d.rec[g].ids[t] = id;
    if (id >= units) bad = true;  // never looked up: the token is refused
    else miss = ld_acq_sys(d.slot_of + base + id) < 0;
  }
  const uint32_t m = __ballot_sync(0xffffffffu, miss), b = __ballot_sync(0xffffffffu, bad);
  if ((t & 31) == 0) {
    mask_w[warp] = m;
    bad_w[warp] = b;
  }
  __syncthreads();
  if (t != 0) return;
  if (bad_w[0] | bad_w[1]) raise(d, kDgBadId, g);
  DgRecord& r = d.rec[g];
  r.n_ids = n;
  r.n_pred_promised = n_pred;
  r.mask_lo = mask_w[0];
  r.mask_hi = mask_w[1];
  r.seq = seq;
  d.any_miss[g] = (mask_w[0] | mask_w[1]) ? 1u : 0u;
  if (d.stamps) {
    volatile unsigned long long* s = d.stamps + 4u * g;
    s[1] = 0ull;
    s[2] = 0ull;
    s[0] = now_ns();
  }
  __threadfence_system();
  st_vol(d.flag + g, seq);
}

__global__ __launch_bounds__(64) void dg_predict_kernel(DgDev d, uint32_t g, const int32_t* ids, uint32_t n) {
  const uint32_t t = threadIdx.x;
  if (t < n) d.prec[g].pred[t] = uint32_t(ids[t]);
  __syncthreads();
  if (t == 0) {
    d.prec[g].n_pred = n;
    __threadfence_system();
    st_vol(d.pflag + g, *d.seq);
  }
}

__global__ void dg_wait_kernel(DgDev d, uint32_t g) {
  if (d.test_flags & kSkipWait) return;
  if (ld_vol(d.abort) || !d.any_miss[g]) return;
  const uint32_t seq = *d.seq;
  const unsigned long long t0 = now_ns();
  if (d.stamps) reinterpret_cast<volatile unsigned long long*>(d.stamps)[4u * g + 1u] = t0;
  for (uint32_t it = 0;; ++it) {
    if (int32_t(ld_acq_gpu(d.ready + g) - seq) >= 0) {
      if (d.stamps) {
        reinterpret_cast<volatile unsigned long long*>(d.stamps)[4u * g + 2u] = now_ns();
        __threadfence_system();
      }
      return;
    }
    if ((it & 15u) == 15u) {
      if (ld_acq_sys(d.host_abort)) {
        raise(d, kDgHostAbort, g);
        return;
      }
      if (now_ns() - t0 > d.timeout_ns) {
        raise(d, kDgTimeout, g);
        return;
      }
    }
    __nanosleep(32);
  }
}

__global__ void dg_end_kernel(DgDev d) {
  if (ld_vol(d.absent_err) && !ld_vol(d.abort)) raise(d, kDgAbsent, 0);
  st_vol(d.m_err_count, *d.err_count);
  st_vol(d.m_err_code, *d.err_code);
  st_vol(d.m_err_aux, *d.err_aux);
  __threadfence_system();
  st_vol(d.done, *d.seq);
}

int last_error() { return int(cudaGetLastError()); }

// A kernel's dynamic shared memory limit is a per-device setting: raised once on each device (bit d of `done`), by
// whichever thread gets there first (setting it twice is harmless).
template <typename K>
int raise_smem_once(K kernel, size_t bytes, std::atomic<uint64_t>& done) {
  int device = 0;
  if (const cudaError_t e = cudaGetDevice(&device); e != cudaSuccess) return int(e);
  const uint64_t bit = device >= 0 && device < 64 ? uint64_t(1) << device : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return 0;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e != cudaSuccess) return int(e);
  done.fetch_or(bit, std::memory_order_acq_rel);
  return 0;
}
std::atomic<uint64_t> g_move_smem_set{0}, g_xxh64_smem_set{0}, g_landed_smem_set{0};

}  // namespace

int launch_batch(const Batch& b, int blocks, void* stream) {
  if (b.n_copies > kMaxCopies || b.n_entries > kMaxEntries) return int(cudaErrorInvalidValue);
  if (blocks < 1) blocks = 1;
  batch_kernel<<<blocks, kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(b);
  return last_error();
}

bool move_fits(const Batch& b) {
  for (uint32_t i = 0; i < b.n_copies; ++i)
    if (((reinterpret_cast<uintptr_t>(b.copies[i].src) | reinterpret_cast<uintptr_t>(b.copies[i].dst) |
          uintptr_t(b.copies[i].bytes)) & 15u) != 0)
      return false;
  return true;
}

int launch_move(const Batch& b, int blocks, void* stream) {
  if (b.n_copies > kMaxCopies || b.n_entries > kMaxEntries || !move_fits(b)) return int(cudaErrorInvalidValue);
  if (const int e = raise_smem_once(move_kernel, kMoveSmem, g_move_smem_set)) return e;
  if (blocks < 1) blocks = 1;
  move_kernel<<<blocks, 32, kMoveSmem, static_cast<cudaStream_t>(stream)>>>(b);
  return last_error();
}

int move_take_timeouts(uint32_t* out) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_move_timeouts, sizeof v);
  if (e == cudaSuccess && v) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_move_timeouts, &zero, sizeof zero);
  }
  *out = v;
  return int(e);
}

int launch_xxh64(const HashUnit* units_dev, uint32_t n, const uint64_t* expect_dev, uint64_t* out_dev,
                 uint32_t* bad_dev, uint32_t* mismatches_dev, void* stream, uint32_t* timeouts_dev) {
  if (!n) return 0;
  if (const int e = raise_smem_once(xxh64_kernel, kHashSmem, g_xxh64_smem_set)) return e;
  const uint32_t blocks = (n + kHashUnits - 1) / kHashUnits;
  xxh64_kernel<<<blocks, 32 * kHashWarps, kHashSmem, static_cast<cudaStream_t>(stream)>>>(
      units_dev, n, expect_dev, out_dev, bad_dev, mismatches_dev, timeouts_dev);
  return last_error();
}

int launch_xxh64_landed(const VerifyBatch& b, void* stream) {
  if (!b.n) return 0;
  if (b.n > kMaxVerify || b.n_parts < 1 || b.n_parts > 4 || !b.expect || !b.bad_count || !b.bad_log ||
      !b.bad_flag || !b.timeouts || !b.done_cnt || !b.done_word)
    return int(cudaErrorInvalidValue);
  if (const int e = raise_smem_once(xxh64_landed_kernel, kHashSmem, g_landed_smem_set)) return e;
  const uint32_t blocks = (b.n + kHashUnits - 1) / kHashUnits;
  xxh64_landed_kernel<<<blocks, 32 * kHashWarps, kHashSmem, static_cast<cudaStream_t>(stream)>>>(b);
  return last_error();
}

int launch_dg_begin(const DgDev& d, void* s) {
  dg_begin_kernel<<<1, 1, 0, static_cast<cudaStream_t>(s)>>>(d);
  return last_error();
}
int launch_dg_export(const DgDev& d, uint32_t g, const int32_t* ids, uint32_t n, uint32_t n_pred, void* s) {
  dg_export_kernel<<<1, 64, 0, static_cast<cudaStream_t>(s)>>>(d, g, ids, n, n_pred);
  return last_error();
}
int launch_dg_predict(const DgDev& d, uint32_t g, const int32_t* ids, uint32_t n, void* s) {
  dg_predict_kernel<<<1, 64, 0, static_cast<cudaStream_t>(s)>>>(d, g, ids, n);
  return last_error();
}
int launch_dg_wait(const DgDev& d, uint32_t g, void* s) {
  dg_wait_kernel<<<1, 1, 0, static_cast<cudaStream_t>(s)>>>(d, g);
  return last_error();
}
int launch_dg_end(const DgDev& d, void* s) {
  dg_end_kernel<<<1, 1, 0, static_cast<cudaStream_t>(s)>>>(d);
  return last_error();
}

int preload() {
  cudaFuncAttributes a;
  const void* fns[] = {(const void*)batch_kernel,      (const void*)xxh64_kernel,     (const void*)xxh64_landed_kernel,
                       (const void*)move_kernel,       (const void*)dg_begin_kernel,  (const void*)dg_export_kernel,
                       (const void*)dg_predict_kernel, (const void*)dg_wait_kernel,   (const void*)dg_end_kernel};
  for (const void* f : fns) {
    const cudaError_t e = cudaFuncGetAttributes(&a, f);
    if (e != cudaSuccess) return int(e);
  }
  if (const int e = raise_smem_once(xxh64_kernel, kHashSmem, g_xxh64_smem_set)) return e;
  if (const int e = raise_smem_once(xxh64_landed_kernel, kHashSmem, g_landed_smem_set)) return e;
  return raise_smem_once(move_kernel, kMoveSmem, g_move_smem_set);
}

int xxh64_take_timeouts(uint32_t* out) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_xxh64_timeouts, sizeof v);
  if (e == cudaSuccess && v) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_xxh64_timeouts, &zero, sizeof zero);
  }
  *out = v;
  return int(e);
}

}  // namespace dev
}  // namespace tsb
