// A minimal stand-in for an inference engine's decode step (tests and bench.py): it drives a device-gated context
// through the public ABI exactly as an engine would. Per token, captured once into a CUDA graph on the caller's
// stream: ss_dg_enqueue_begin, then per gated layer ss_dg_enqueue_export of that layer's routed ids (read from a device
// buffer the host refills before each launch), ss_dg_enqueue_wait, and a reader kernel that resolves every id through
// ss_dg_slot (the engine-side inline of ss.h) and reads the whole unit, as a batch-1 MoE matvec reads its experts;
// then ss_dg_enqueue_end. The reader's result per (layer, id) is a checksum of the unit's bytes:
//   mode 0: sum(byte * (pos % 251 + 1)) over the unit (the reference GPU tests' check, tests/test_dg_cuda.cu:103-114);
//   mode 1: the sum of the unit's 32-bit little-endian words (a read at HBM speed, the bench's engine work).
// This library is not part of the runtime (libtierstream.so never links it).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "strix_stream/ss.h"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint64_t warp_sum(uint64_t v) {
  for (int o = 16; o; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;
}

// sum over k < 16 of byte k x ((m + k) % 251 + 1) for the 16 bytes of w (m < 251): (m + 1) x sum(b) + sum(k x b) from
// byte dot products, less 251 x b for the bytes past the wrap (k >= 251 - m, only when m > 235).
__device__ __forceinline__ uint64_t weighted16(const uint4& w, uint32_t m) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
  uint32_t s0 = 0, s1 = 0;
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    s0 = __dp4a(words[j], 0x01010101u, s0);
    s1 = __dp4a(words[j], 0x03020100u + 0x04040404u * j, s1);
  }
  uint64_t v = uint64_t(m + 1) * s0 + s1;
  if (m > 235)
    for (uint32_t k = 251 - m; k < 16; ++k) v -= 251ull * ((words[k >> 2] >> (8 * (k & 3))) & 0xffu);
  return v;
}

// The checksum contribution of one 16-byte group at unit position 16 x e (m = that position % 251).
__device__ __forceinline__ uint64_t group_sum(const uint4& w, uint32_t m, int mode) {
  return mode == 1 ? uint64_t(w.x) + w.y + w.z + w.w : weighted16(w, m);
}

// grid (n, slices): block (i, s) reads slice s of unit ids[i] of gated layer g and adds its part of the checksum. A
// slice is a range of the unit's 16-byte groups (its parts back to back); each part it covers is walked directly, four
// 16-byte loads in flight per thread.
__global__ __launch_bounds__(kThreads) void reader_kernel(ss_dg_device_view v, uint32_t g, const int32_t* ids,
                                                          uint32_t n, unsigned long long* out, int mode) {
  const uint32_t i = blockIdx.x;
  if (i >= n) return;
  const int32_t slot = ss_dg_slot(&v, g, ids[i]);
  uint64_t n16 = 0;
  for (uint32_t p = 0; p < v.n_parts; ++p) n16 += v.parts[p].bytes / 16;  // every part is a multiple of 256 bytes
  const uint64_t per = (n16 + gridDim.y - 1) / gridDim.y;
  const uint64_t lo = per * blockIdx.y, hi = lo + per < n16 ? lo + per : n16;
  constexpr uint32_t kStep = (16u * kThreads) % 251u;  // m advances by this per kThreads groups
  uint64_t acc = 0, first = 0;
  for (uint32_t p = 0; p < v.n_parts; ++p) {
    const uint64_t len = v.parts[p].bytes / 16;
    const uint64_t a = lo > first ? lo : first, b = hi < first + len ? hi : first + len;
    if (a < b) {
      const uint4* base = reinterpret_cast<const uint4*>(static_cast<const char*>(v.parts[p].base) +
                                                         uint64_t(slot) * v.parts[p].stride) - first;
      uint64_t e = a + threadIdx.x;
      uint32_t m = uint32_t((e * 16) % 251);
      for (; e + 3 * kThreads < b; e += 4 * kThreads) {
        uint4 w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) w[k] = base[e + uint64_t(k) * kThreads];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc += group_sum(w[k], m, mode);
          m += kStep;
          if (m >= 251) m -= 251;
        }
      }
      for (; e < b; e += kThreads) {
        acc += group_sum(base[e], m, mode);
        m += kStep;
        if (m >= 251) m -= 251;
      }
    }
    first += len;
  }
  __shared__ uint64_t part[kThreads / 32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t s = 0;
    for (int k = 0; k < kThreads / 32; ++k) s += part[k];
    atomicAdd(out + i, (unsigned long long)s);
  }
}

// Host forward mode's reader: unit ids[i] at the address table_dev[ids[i]] (ss_layer_view.table_dev), unit_bytes
// long; the positional checksum of tests/test_cuda.cu's checksum kernel (64-75 there). A zero address reads as 0.
__global__ __launch_bounds__(kThreads) void table_reader_kernel(const uint64_t* table, const int32_t* ids, uint32_t n,
                                                                uint64_t unit_bytes, unsigned long long* out) {
  const uint32_t i = blockIdx.x;
  if (i >= n) return;
  const uint8_t* base = reinterpret_cast<const uint8_t*>(table[ids[i]]);
  uint64_t acc = 0;
  if (base) {
    const uint64_t per = (unit_bytes + gridDim.y - 1) / gridDim.y;
    const uint64_t lo = per * blockIdx.y, hi = lo + per < unit_bytes ? lo + per : unit_bytes;
    for (uint64_t p = lo + threadIdx.x; p < hi; p += kThreads) acc += uint64_t(base[p]) * (p % 251 + 1);
  }
  __shared__ uint64_t part[kThreads / 32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t s = 0;
    for (int k = 0; k < kThreads / 32; ++k) s += part[k];
    atomicAdd(out + i, (unsigned long long)s);
  }
}

// Host forward mode's reader for units whose bytes are a multiple of 16 at 16-byte aligned addresses (every pinned
// and device slot is): the same checksums as reader_kernel's modes, 16-byte loads, four in flight per thread.
__global__ __launch_bounds__(kThreads) void table_reader16_kernel(const uint64_t* table, const int32_t* ids, uint32_t n,
                                                                  uint64_t unit_bytes, unsigned long long* out,
                                                                  int mode) {
  const uint32_t i = blockIdx.x;
  if (i >= n) return;
  const uint4* base = reinterpret_cast<const uint4*>(table[ids[i]]);
  uint64_t acc = 0;
  if (base) {
    const uint64_t n16 = unit_bytes / 16;
    const uint64_t per = (n16 + gridDim.y - 1) / gridDim.y;
    const uint64_t lo = per * blockIdx.y, hi = lo + per < n16 ? lo + per : n16;
    constexpr uint32_t kStep = (16u * kThreads) % 251u;
    uint64_t e = lo + threadIdx.x;
    uint32_t m = uint32_t((e * 16) % 251);
    for (; e + 3 * kThreads < hi; e += 4 * kThreads) {
      uint4 w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) w[k] = base[e + uint64_t(k) * kThreads];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc += group_sum(w[k], m, mode);
        m += kStep;
        if (m >= 251) m -= 251;
      }
    }
    for (; e < hi; e += kThreads) {
      acc += group_sum(base[e], m, mode);
      m += kStep;
      if (m >= 251) m -= 251;
    }
  }
  __shared__ uint64_t part[kThreads / 32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t s = 0;
    for (int k = 0; k < kThreads / 32; ++k) s += part[k];
    atomicAdd(out + i, (unsigned long long)s);
  }
}

#define CK(x)                                  \
  do {                                         \
    const cudaError_t e_ = (x);                \
    if (e_ != cudaSuccess) return int(e_);     \
  } while (0)
#define SS(x)                                  \
  do {                                         \
    const ss_status s_ = (x);                  \
    if (s_ != SS_OK) return 1000 + int(s_);    \
  } while (0)

}  // namespace

extern "C" {

// Captures one token step into a graph on `stream`: for gated layer g its n_ids ids are ids_dev[g * n_ids ..], its
// results out_dev[g * n_ids ..] (zeroed by the graph first). slices: blocks per unit for the reader. n_pred > 0: each
// layer g < G - 1 also predicts layer g + 1 from pred_dev[g * n_pred ..] on a forked branch joined before the next
// export. held (host, n_gated flags, may be NULL): layers held resident by ss_dg_make_resident, which an engine
// neither exports nor waits for: their reader resolves the ids through the table directly (a layer before a held one
// predicts nothing). Returns 0 or an error (cudaError_t, or 1000 + ss_status) and the instantiated graph in *exec_out.
__attribute__((visibility("default"))) int tse_capture_token(ss_ctx* c, uint32_t n_gated, const int32_t* ids_dev,
                                                             uint32_t n_ids, const int32_t* pred_dev, uint32_t n_pred,
                                                             unsigned long long* out_dev, uint32_t slices, int mode,
                                                             int with_reader, void* stream, void** exec_out,
                                                             const uint8_t* held) {
  ss_dg_device_view v;
  SS(ss_dg_get_device_view(c, &v));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  if (n_pred) {
    CK(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&fork, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&join, cudaEventDisableTiming));
  }
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
  int err = 0;
  do {
    if (with_reader && cudaMemsetAsync(out_dev, 0, size_t(n_gated) * n_ids * 8, s) != cudaSuccess) {
      err = 1;
      break;
    }
    if (ss_dg_enqueue_begin(c, s) != SS_OK) {
      err = 1001;
      break;
    }
    for (uint32_t g = 0; g < n_gated && !err; ++g) {
      const bool is_held = held && held[g];
      const int np = (n_pred && g + 1 < n_gated && !(held && held[g + 1])) ? int(n_pred) : 0;
      if (!is_held && ss_dg_enqueue_export(c, int(g), ids_dev + size_t(g) * n_ids, int(n_ids), np, s) != SS_OK)
        err = 1002;
      if (!err && np && !is_held) {
        if (cudaEventRecord(fork, s) != cudaSuccess || cudaStreamWaitEvent(side, fork, 0) != cudaSuccess) err = 2;
        if (!err && ss_dg_enqueue_predict(c, int(g), pred_dev + size_t(g) * n_pred, np, side) != SS_OK) err = 1003;
      }
      if (!err && !is_held && ss_dg_enqueue_wait(c, int(g), s) != SS_OK) err = 1004;
      if (!err && with_reader) {
        reader_kernel<<<dim3(n_ids, slices), kThreads, 0, s>>>(v, g, ids_dev + size_t(g) * n_ids, n_ids,
                                                              out_dev + size_t(g) * n_ids, mode);
        if (cudaGetLastError() != cudaSuccess) err = 3;
      }
      if (!err && np && !is_held) {
        if (cudaEventRecord(join, side) != cudaSuccess || cudaStreamWaitEvent(s, join, 0) != cudaSuccess) err = 4;
      }
    }
    if (!err && ss_dg_enqueue_end(c, s) != SS_OK) err = 1005;
  } while (false);
  const cudaError_t ec = cudaStreamEndCapture(s, &graph);
  if (side) cudaStreamDestroy(side);
  if (fork) cudaEventDestroy(fork);
  if (join) cudaEventDestroy(join);
  if (err) {
    if (graph) cudaGraphDestroy(graph);
    return err;
  }
  CK(ec);
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  CK(ei);
  *exec_out = exec;
  return 0;
}

// The synthetic byte stream of the benchmark's model files: byte i of file `file_id` (the reference fixtures'
// generator, tests/fixture.hpp:16-22), n bytes from position `first`, on `threads` host threads.
__attribute__((visibility("default"))) void tse_fill_bytes(uint64_t file_id, uint64_t first, uint64_t n, uint8_t* out,
                                                           uint32_t threads) {
  if (threads < 1) threads = 1;
  auto fill = [=](uint64_t lo, uint64_t hi) {
    for (uint64_t j = lo; j < hi; ++j) {
      const uint64_t i = first + j;
      uint64_t x = (i + 1) * 0x9E3779B97F4A7C15ULL ^ (file_id + 7) * 0xC2B2AE3D27D4EB4FULL;
      x ^= x >> 29;
      x *= 0xBF58476D1CE4E5B9ULL;
      x ^= x >> 32;
      out[j] = uint8_t(x);
    }
  };
  std::vector<std::thread> th;
  const uint64_t per = (n + threads - 1) / threads;
  for (uint32_t t = 0; t < threads; ++t) {
    const uint64_t lo = per * t, hi = lo + per < n ? lo + per : n;
    if (lo < hi) th.emplace_back(fill, lo, hi);
  }
  for (auto& t : th) t.join();
}

// Byte i of file `file_id` of the synthetic stream (the same formula as tse_fill_bytes), on the device.
__device__ __forceinline__ uint8_t gen_byte(uint64_t file_id, uint64_t i) {
  uint64_t x = (i + 1) * 0x9E3779B97F4A7C15ULL ^ (file_id + 7) * 0xC2B2AE3D27D4EB4FULL;
  x ^= x >> 29;
  x *= 0xBF58476D1CE4E5B9ULL;
  x ^= x >> 32;
  return uint8_t(x);
}

// The same byte stream written on the device: n bytes of file `file_id` from position `first` into dst (HBM), for a
// store the caller fills itself (tsb_peer_store_alloc) without a model file on disk.
__global__ void fill_bytes_kernel(uint64_t file_id, uint64_t first, uint64_t n, uint8_t* __restrict__ dst) {
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x * 8;
  for (uint64_t j = (uint64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 8; j < n; j += stride) {
    uint64_t word = 0;
    const uint64_t m = n - j < 8 ? n - j : 8;
    for (uint64_t k = 0; k < m; ++k) word |= uint64_t(gen_byte(file_id, first + j + k)) << (8 * k);
    if (m == 8 && ((reinterpret_cast<uintptr_t>(dst + j) & 7u) == 0)) {
      *reinterpret_cast<uint64_t*>(dst + j) = word;
    } else {
      for (uint64_t k = 0; k < m; ++k) dst[j + k] = uint8_t(word >> (8 * k));
    }
  }
}

// The reader's checksum of unit i (unit_bytes from file position offsets[i]) computed from the byte generator alone,
// never from a copy: grid (n, slices), each block a slice of the unit's 16-byte groups, in reader_kernel's modes
// (0: sum(byte x (pos % 251 + 1)), 1: the sum of the unit's 32-bit little-endian words). unit_bytes % 16 == 0.
__global__ __launch_bounds__(kThreads) void expect_sums_kernel(uint64_t file_id, const uint64_t* offsets,
                                                               uint64_t unit_bytes, int mode,
                                                               unsigned long long* out) {
  const uint32_t i = blockIdx.x;
  const uint64_t base = offsets[i];
  const uint64_t n16 = unit_bytes / 16;
  const uint64_t per = (n16 + gridDim.y - 1) / gridDim.y;
  const uint64_t lo = per * blockIdx.y, hi = lo + per < n16 ? lo + per : n16;
  uint64_t acc = 0;
  for (uint64_t e = lo + threadIdx.x; e < hi; e += kThreads) {
    const uint64_t pos = e * 16;
    uint32_t m = uint32_t(pos % 251);
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint64_t b = gen_byte(file_id, base + pos + uint64_t(k));
      if (mode == 1) {
        acc += b << (8 * (k & 3));
      } else {
        acc += b * (m + 1);
        m = m + 1 == 251 ? 0 : m + 1;
      }
    }
  }
  __shared__ uint64_t part[kThreads / 32];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t s = 0;
    for (int k = 0; k < kThreads / 32; ++k) s += part[k];
    atomicAdd(out + i, (unsigned long long)s);
  }
}

// n units: unit i's bytes (unit_bytes from file position offsets[i]) into dst + i * unit_bytes, on `stream`.
__attribute__((visibility("default"))) int tse_fill_units_device(uint64_t file_id, const uint64_t* offsets, uint32_t n,
                                                                 uint64_t unit_bytes, void* dst, void* stream) {
  for (uint32_t i = 0; i < n; ++i) {
    fill_bytes_kernel<<<592, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        file_id, offsets[i], unit_bytes, static_cast<uint8_t*>(dst) + uint64_t(i) * unit_bytes);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return int(e);
  }
  return 0;
}

// Expected reader checksums of n units from the generator (expect_sums_kernel): offsets_dev[n] (device) the units'
// file positions, out_dev[n] (device) zeroed here first, on `stream`.
__attribute__((visibility("default"))) int tse_expect_sums(uint64_t file_id, const uint64_t* offsets_dev, uint32_t n,
                                                           uint64_t unit_bytes, int mode, unsigned long long* out_dev,
                                                           uint32_t slices, void* stream) {
  if (!n) return 0;
  if (unit_bytes % 16 != 0 || (mode != 0 && mode != 1)) return int(cudaErrorInvalidValue);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemsetAsync(out_dev, 0, size_t(n) * 8, s));
  expect_sums_kernel<<<dim3(n, slices ? slices : 1), kThreads, 0, s>>>(file_id, offsets_dev, unit_bytes, mode, out_dev);
  return int(cudaGetLastError());
}

__attribute__((visibility("default"))) int tse_launch(void* exec, void* stream) {
  return int(cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), static_cast<cudaStream_t>(stream)));
}

__attribute__((visibility("default"))) int tse_destroy(void* exec) {
  return int(cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec)));
}

// Host forward mode: checksums of n units read through an acquired layer's device address table, on `stream`.
__attribute__((visibility("default"))) int tse_read_table(const uint64_t* table_dev, const int32_t* ids_dev,
                                                          uint32_t n, uint64_t unit_bytes,
                                                          unsigned long long* out_dev, uint32_t slices, void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemsetAsync(out_dev, 0, size_t(n) * 8, s));
  table_reader_kernel<<<dim3(n, slices), kThreads, 0, s>>>(table_dev, ids_dev, n, unit_bytes, out_dev);
  return int(cudaGetLastError());
}

// Host forward mode with 16-byte loads (unit_bytes a multiple of 16): mode 0 the positional checksum (as
// tse_read_table), mode 1 the 32-bit word sum; on `stream`.
__attribute__((visibility("default"))) int tse_read_table16(const uint64_t* table_dev, const int32_t* ids_dev,
                                                            uint32_t n, uint64_t unit_bytes,
                                                            unsigned long long* out_dev, uint32_t slices, int mode,
                                                            void* stream) {
  if (unit_bytes % 16 != 0 || (mode != 0 && mode != 1)) return int(cudaErrorInvalidValue);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemsetAsync(out_dev, 0, size_t(n) * 8, s));
  table_reader16_kernel<<<dim3(n, slices ? slices : 1), kThreads, 0, s>>>(table_dev, ids_dev, n, unit_bytes, out_dev,
                                                                          mode);
  return int(cudaGetLastError());
}

// One host-mode forward of an engine over descriptor d, all of it native: ss_begin; per layer with units, its routes (ss_layer_routes
// of routes[L][0..n_ids), or ss_layer_all when all_layers[L] != 0), ss_acquire on `stream`, the reader over the
// layer's ids (the routed ids, or unit 0 for a whole layer) through the acquired device table, ss_release; ss_end.
// ids_dev [layers][n_ids] (device) receives the token's ids by one copy from `routes` (pinned host memory for an
// asynchronous copy) at the start; out_dev [layers][n_ids] the readers' checksums (mode 0 positional, 1 word sums;
// 16-byte loads when unit_bytes % 16 == 0, else the byte reader, mode 0 only). Returns 0, a CUDA error, or
// 1000 + an ss_status.
__attribute__((visibility("default"))) int tse_host_forward(ss_ctx* c, const ss_desc* d, const int32_t* routes,
                                                            uint32_t n_ids,
                                                            const uint8_t* all_layers, int32_t* ids_dev,
                                                            unsigned long long* out_dev, uint32_t slices, int mode,
                                                            void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int layers = ss_desc_n_layers(d);
  if (layers < 0) return 1000 + int(SS_E_INVALID);
  CK(cudaMemcpyAsync(ids_dev, routes, sizeof(int32_t) * size_t(layers) * n_ids, cudaMemcpyHostToDevice, s));
  CK(cudaMemsetAsync(out_dev, 0, sizeof(unsigned long long) * size_t(layers) * n_ids, s));
  SS(ss_begin(c, nullptr, 0));
  for (int L = 0; L < layers; ++L) {
    const int units = ss_desc_layer_units(d, L);
    if (units <= 0) continue;
    const bool whole = all_layers && all_layers[L];
    if (whole) SS(ss_layer_all(c, L));
    else SS(ss_layer_routes(c, L, routes + size_t(L) * n_ids, int(n_ids)));
    ss_layer_view v;
    SS(ss_acquire(c, L, stream, &v));
    const uint64_t unit_bytes = ss_desc_unit_bytes(d, L);
    const uint32_t n = whole ? 1u : n_ids;
    int32_t* ids = ids_dev + size_t(L) * n_ids;
    unsigned long long* out = out_dev + size_t(L) * n_ids;
    if (unit_bytes % 16 == 0) {
      table_reader16_kernel<<<dim3(n, slices ? slices : 1), kThreads, 0, s>>>(v.table_dev, ids, n, unit_bytes, out,
                                                                              mode);
    } else {
      if (mode != 0) return int(cudaErrorInvalidValue);
      table_reader_kernel<<<dim3(n, slices ? slices : 1), kThreads, 0, s>>>(v.table_dev, ids, n, unit_bytes, out);
    }
    CK(cudaGetLastError());
    SS(ss_release(c, L, stream));
  }
  SS(ss_end(c));
  return 0;
}

// The reader alone (no capture): checksums of n units of gated layer g resolved through the context's table.
__attribute__((visibility("default"))) int tse_read_units(ss_ctx* c, uint32_t g, const int32_t* ids_dev, uint32_t n,
                                                          unsigned long long* out_dev, uint32_t slices, int mode,
                                                          void* stream) {
  ss_dg_device_view v;
  SS(ss_dg_get_device_view(c, &v));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CK(cudaMemsetAsync(out_dev, 0, size_t(n) * 8, s));
  reader_kernel<<<dim3(n, slices), kThreads, 0, s>>>(v, g, ids_dev, n, out_dev, mode);
  return int(cudaGetLastError());
}

}  // extern "C"
