// Device kernels of the B200 runtime (sm_100a). Byte movement and control only: no tensor-core work exists on this
// path. See kernels.hpp for the launch contracts.
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.hpp"

namespace tsb {
namespace dev {
namespace {

// ---------------------------------------------------------------------------------------------------------------
// K1 / K4 / K5: the batched copy ("land") kernel.
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
// K3: xxh64 of whole units. One lane quad per unit: lane l carries accumulator l. A warp serves 8 units and stages
// their bytes through shared memory with cp.async (8 stages x 1 KiB per unit), so the serial lane chains never wait
// on HBM. Units whose spans are not 32-byte multiples (except the last) or not 16-byte aligned take a one-lane path.
// ---------------------------------------------------------------------------------------------------------------
constexpr uint64_t X1 = 0x9E3779B185EBCA87ULL, X2 = 0xC2B2AE3D27D4EB4FULL, X3 = 0x165667B19E3779F9ULL,
                   X4 = 0x85EBCA77C2B2AE63ULL, X5 = 0x27D4EB2F165667C5ULL;
constexpr int kHashUnits = 8, kHashStages = 8, kHashChunk = 1024;

__device__ __forceinline__ uint64_t rotl64(uint64_t v, uint32_t r) { return (v << r) | (v >> (64 - r)); }
__device__ __forceinline__ uint64_t lane_step(uint64_t acc, uint64_t w) { return rotl64(acc + w * X2, 31) * X1; }

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

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = uint32_t(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__global__ __launch_bounds__(32) void xxh64_kernel(const HashUnit* __restrict__ units, uint32_t n,
                                                   const uint64_t* __restrict__ expect, uint64_t* __restrict__ out,
                                                   uint32_t* __restrict__ bad, uint32_t* __restrict__ mismatches) {
  extern __shared__ __align__(16) uint8_t stage_buf[];  // [kHashUnits][kHashStages][kHashChunk]
  const uint32_t lane = threadIdx.x, q = lane >> 2, l = lane & 3;
  const uint32_t first = blockIdx.x * kHashUnits;
  // per unit of this warp: its stripe bytes (0 for the one-lane path) and total bytes
  uint64_t body[kHashUnits], total[kHashUnits];
  bool fast[kHashUnits];
  uint32_t nchunks = 0;
#pragma unroll
  for (int i = 0; i < kHashUnits; ++i) {
    body[i] = total[i] = 0;
    fast[i] = false;
    if (first + i >= n) continue;
    const HashUnit& u = units[first + i];
    bool ok = u.n_spans >= 1 && u.n_spans <= 4;
    uint64_t t = 0;
    for (uint32_t s = 0; ok && s < u.n_spans; ++s) {
      ok = (reinterpret_cast<uintptr_t>(u.span[s]) & 15u) == 0 && (s + 1 == u.n_spans || u.bytes[s] % 32 == 0);
      t += u.bytes[s];
    }
    if (!ok) {
      t = 0;
      for (uint32_t s = 0; s < u.n_spans && s < 4; ++s) t += u.bytes[s];
    }
    total[i] = t;
    fast[i] = ok;
    body[i] = ok ? t / 32 * 32 : 0;
    const uint32_t c = uint32_t((body[i] + kHashChunk - 1) / kHashChunk);
    nchunks = c > nchunks ? c : nchunks;
  }
  // issue chunk c of every unit: 8 units x 64 vectors, 16 per lane
  auto issue = [&](uint32_t c) {
    const size_t stage_off = size_t(c % kHashStages) * kHashChunk;
#pragma unroll 4
    for (uint32_t e = lane; e < kHashUnits * (kHashChunk / 16); e += 32) {
      const uint32_t i = e / (kHashChunk / 16), v = e % (kHashChunk / 16);
      uint64_t p = uint64_t(c) * kHashChunk + uint64_t(v) * 16;
      if (p >= body[i]) continue;
      const HashUnit& u = units[first + i];
      uint32_t s = 0;
      while (p >= u.bytes[s]) {
        p -= u.bytes[s];
        ++s;
      }
      cp_async16(stage_buf + size_t(i) * kHashStages * kHashChunk + stage_off + size_t(v) * 16, u.span[s] + p);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  uint64_t acc = l == 0 ? X1 + X2 : l == 1 ? X2 : l == 2 ? 0 : uint64_t(0) - X1;  // seed 0
  for (uint32_t c = 0; c + 1 < kHashStages; ++c) {
    if (c < nchunks) issue(c);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (uint32_t c = 0; c < nchunks; ++c) {
    if (c + kHashStages - 1 < nchunks) issue(c + kHashStages - 1);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group %0;" ::"n"(kHashStages - 1) : "memory");
    __syncwarp();
    const uint64_t start = uint64_t(c) * kHashChunk;
    if (start < body[q]) {
      const uint64_t left = body[q] - start;
      const uint32_t stripes = left >= kHashChunk ? kHashChunk / 32 : uint32_t(left / 32);
      const uint64_t* w = reinterpret_cast<const uint64_t*>(stage_buf + size_t(q) * kHashStages * kHashChunk +
                                                            size_t(c % kHashStages) * kHashChunk) + l;
#pragma unroll 8
      for (uint32_t s = 0; s < stripes; ++s) acc = lane_step(acc, w[4 * s]);
    }
    __syncwarp();
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  // gather the quad's accumulators on its lane 0
  uint64_t v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = __shfl_sync(0xffffffffu, acc, int((lane & ~3u) + k));
  const uint32_t idx = first + q;
  if (l != 0 || idx >= n) return;
  const HashUnit& u = units[idx];
  uint64_t h;
  if (fast[q]) {
    h = finish_hash(u, v, total[q], body[q]);
  } else {  // one lane: the stripes from global memory
    uint64_t a[4] = {X1 + X2, X2, 0, uint64_t(0) - X1};
    const uint64_t b = total[q] / 32 * 32;
    for (uint64_t p = 0; p < b; p += 32)
      for (int k = 0; k < 4; ++k) a[k] = lane_step(a[k], unit_le64(u, p + 8 * uint64_t(k)));
    h = finish_hash(u, a, total[q], b);
  }
  out[idx] = h;
  if (expect && expect[idx] != h) {
    if (bad) bad[idx] = 1;
    if (mismatches) atomicAdd(mismatches, 1u);
  }
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

}  // namespace

int launch_batch(const Batch& b, int blocks, void* stream) {
  if (b.n_copies > kMaxCopies || b.n_entries > kMaxEntries) return int(cudaErrorInvalidValue);
  if (blocks < 1) blocks = 1;
  batch_kernel<<<blocks, kCopyThreads, 0, static_cast<cudaStream_t>(stream)>>>(b);
  return last_error();
}

int launch_xxh64(const HashUnit* units_dev, uint32_t n, const uint64_t* expect_dev, uint64_t* out_dev,
                 uint32_t* bad_dev, uint32_t* mismatches_dev, void* stream) {
  if (!n) return 0;
  const size_t smem = size_t(kHashUnits) * kHashStages * kHashChunk;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(xxh64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return int(e);
    attr = true;
  }
  const uint32_t blocks = (n + kHashUnits - 1) / kHashUnits;
  xxh64_kernel<<<blocks, 32, smem, static_cast<cudaStream_t>(stream)>>>(units_dev, n, expect_dev, out_dev, bad_dev,
                                                                        mismatches_dev);
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
  const void* fns[] = {(const void*)batch_kernel,     (const void*)xxh64_kernel,      (const void*)dg_begin_kernel,
                       (const void*)dg_export_kernel, (const void*)dg_predict_kernel, (const void*)dg_wait_kernel,
                       (const void*)dg_end_kernel};
  for (const void* f : fns) {
    const cudaError_t e = cudaFuncGetAttributes(&a, f);
    if (e != cudaSuccess) return int(e);
  }
  const size_t smem = size_t(kHashUnits) * kHashStages * kHashChunk;
  return int(cudaFuncSetAttribute(xxh64_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
}

}  // namespace dev
}  // namespace tsb
