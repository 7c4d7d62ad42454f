// The tsb_* entry points of include/tierstream/tsb.h.
#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "dg_core.hpp"
#include "errors.hpp"
#include "kernels.hpp"
#include "source_file.hpp"
#include "tierstream/tsb.h"
#include "xxh64.hpp"

namespace tsb {
void dg_replay(const tsb_dg_replay_config* c, const int32_t* ids, const int32_t* preds, int32_t* tables,
               uint64_t* stats, const uint8_t* src_units, uint64_t* read_sum);
const char* set_error(const std::string& msg);
}  // namespace tsb

namespace {

template <class F>
ss_status run(F&& f) {
  try {
    f();
    return SS_OK;
  } catch (const tsb::Error& e) {
    tsb::set_error(e.what());
    return e.status();
  } catch (const std::exception& e) {
    tsb::set_error(e.what());
    return SS_E_BACKEND;
  }
}
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    tsb::fail(SS_E_BACKEND, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

}  // namespace

namespace {
ss_status land_or_move(bool move, const void* const* src, void* const* dst, const uint64_t* bytes, uint32_t n,
                       int32_t* slot_of, const uint32_t* keys, const int32_t* vals, uint32_t n_entries,
                       uint32_t* ready_word, uint32_t ready_val, uint32_t* counter, uint32_t blocks, void* stream) {
  return run([&] {
    tsb::require(n <= tsb::dev::kMaxCopies && n_entries <= tsb::dev::kMaxEntries, SS_E_INVALID,
                 "tsb_land: at most 384 copies and 128 entries per call");
    tsb::require((!n || (src && dst && bytes)) && (!n_entries || (slot_of && keys && vals)), SS_E_INVALID,
                 "tsb_land: null argument");
    tsb::require(counter || (!n_entries && !ready_word), SS_E_INVALID,
                 "tsb_land: publishing entries or a ready word needs a counter word");
    auto b = std::make_unique<tsb::dev::Batch>();
    b->n_copies = n;
    b->n_entries = n_entries;
    b->slot_of = slot_of;
    b->ready_word = ready_word;
    b->ready_val = ready_val;
    b->done_counter = counter;
    uint64_t chunks = 0;
    for (uint32_t i = 0; i < n; ++i) {
      b->copies[i] = {src[i], dst[i], bytes[i]};
      chunks += (bytes[i] + (64u << 10) - 1) >> 16;
    }
    for (uint32_t i = 0; i < n_entries; ++i) {
      b->entry_key[i] = keys[i];
      b->entry_val[i] = vals[i];
    }
    if (move) {
      tsb::require(tsb::dev::move_fits(*b), SS_E_INVALID,
                   "tsb_move: every address and size must be a multiple of 16 bytes (TMA bulk copies)");
      const int grid = blocks ? int(blocks) : int(chunks < 1 ? 1 : chunks > 148 ? 148 : chunks);
      ck(cudaError_t(tsb::dev::launch_move(*b, grid, stream)), "move kernel");
      return;
    }
    const int grid = blocks ? int(blocks) : int(chunks < 1 ? 1 : chunks > 296 ? 296 : chunks);
    ck(cudaError_t(tsb::dev::launch_batch(*b, grid, stream)), "land kernel");
  });
}
}  // namespace

extern "C" {

ss_status tsb_land(const void* const* src, void* const* dst, const uint64_t* bytes, uint32_t n, int32_t* slot_of,
                   const uint32_t* keys, const int32_t* vals, uint32_t n_entries, uint32_t* ready_word,
                   uint32_t ready_val, uint32_t* counter, uint32_t blocks, void* stream) {
  return land_or_move(false, src, dst, bytes, n, slot_of, keys, vals, n_entries, ready_word, ready_val, counter,
                      blocks, stream);
}

ss_status tsb_move(const void* const* src, void* const* dst, const uint64_t* bytes, uint32_t n, int32_t* slot_of,
                   const uint32_t* keys, const int32_t* vals, uint32_t n_entries, uint32_t* ready_word,
                   uint32_t ready_val, uint32_t* counter, uint32_t blocks, void* stream) {
  return land_or_move(true, src, dst, bytes, n, slot_of, keys, vals, n_entries, ready_word, ready_val, counter,
                      blocks, stream);
}

int tsb_move_timeouts(void) {
  uint32_t v = 0;
  return tsb::dev::move_take_timeouts(&v) == 0 ? int(v) : -1;
}

ss_status tsb_xxh64_units(const void* const* spans, const uint64_t* span_bytes, const uint32_t* n_spans, uint32_t n,
                          void* units_dev, const uint64_t* expect_dev, uint64_t* out_dev, uint32_t* mismatches_dev,
                          void* stream) {
  return run([&] {
    if (!n) return;
    tsb::require(spans && span_bytes && n_spans && units_dev && out_dev, SS_E_INVALID, "tsb_xxh64_units: null argument");
    tsb::require(!expect_dev || mismatches_dev, SS_E_INVALID, "tsb_xxh64_units: expected hashes need a mismatch word");
    std::vector<tsb::dev::HashUnit> u(n);
    for (uint32_t i = 0; i < n; ++i) {
      tsb::require(n_spans[i] >= 1 && n_spans[i] <= 4, SS_E_INVALID, "tsb_xxh64_units: 1..4 spans per unit");
      u[i] = tsb::dev::HashUnit{};
      u[i].n_spans = n_spans[i];
      for (uint32_t s = 0; s < n_spans[i]; ++s) {
        u[i].span[s] = static_cast<const uint8_t*>(spans[4 * size_t(i) + s]);
        u[i].bytes[s] = span_bytes[4 * size_t(i) + s];
      }
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ck(cudaMemcpyAsync(units_dev, u.data(), u.size() * sizeof(tsb::dev::HashUnit), cudaMemcpyHostToDevice, s),
       "tsb_xxh64_units: unit table upload");
    ck(cudaError_t(tsb::dev::launch_xxh64(static_cast<const tsb::dev::HashUnit*>(units_dev), n, expect_dev, out_dev,
                                          nullptr, mismatches_dev, s)),
       "xxh64 kernel");
    ck(cudaStreamSynchronize(s), "tsb_xxh64_units: sync");  // the host unit table is released on return
    uint32_t timeouts = 0;
    ck(cudaError_t(tsb::dev::xxh64_take_timeouts(&timeouts)), "tsb_xxh64_units: timeout word");
    tsb::require(!timeouts, SS_E_BACKEND, "tsb_xxh64_units: a staging copy of the xxh64 kernel did not complete");
  });
}

ss_status tsb_test_dg_replay(const tsb_dg_replay_config* cfg, const int32_t* ids, const int32_t* preds,
                             int32_t* tables, uint64_t* stats, const uint8_t* src_units, uint64_t* read_sum) {
  return run([&] { tsb::dg_replay(cfg, ids, preds, tables, stats, src_units, read_sum); });
}

ss_status tsb_test_file_read(const char* path, uint64_t offset, uint64_t bytes, void* dst, uint64_t piece,
                             uint32_t threads, int direct) {
  return run([&] {
    tsb::require(path && (dst || !bytes) && piece >= 1 && threads >= 1 && threads <= 64, SS_E_INVALID,
                 "tsb_test_file_read: bad argument");
    tsb::SourceFile f(path, 4096, direct != 0);
    tsb::ReadPool pool(threads);
    const uint64_t n = (bytes + piece - 1) / piece;
    pool.run(size_t(n), [&](size_t i) {
      const uint64_t o = uint64_t(i) * piece;
      f.read(static_cast<char*>(dst) + o, offset + o, std::min(piece, bytes - o));
    });
  });
}

ss_status tsb_test_async_reads(const char* path, const uint64_t* offsets, uint32_t n, uint64_t bytes, void* dst,
                               uint32_t threads, int reverse) {
  return run([&] {
    tsb::require(path && (offsets || !n) && (dst || !n) && threads >= 1 && threads <= 64, SS_E_INVALID,
                 "tsb_test_async_reads: bad argument");
    tsb::SourceFile f(path, 4096, true);
    tsb::AsyncReads q(threads, [&](uint32_t i, char* out) { f.read(out, offsets[i], bytes); });
    std::vector<void*> h(n);
    for (uint32_t i = 0; i < n; ++i) h[i] = q.begin(i, static_cast<char*>(dst) + uint64_t(i) * bytes);
    std::exception_ptr first;
    for (uint32_t k = 0; k < n; ++k) {
      const uint32_t i = reverse ? n - 1 - k : k;
      try {
        q.end(h[i]);
      } catch (...) {
        if (!first) first = std::current_exception();
      }
    }
    if (first) std::rethrow_exception(first);
  });
}

uint64_t tsb_xxh64(const void* data, size_t len, uint64_t seed) { return tsb::xxh64(data, len, seed); }

int tsb_cuda_arch(void) { return 100; }

}  // extern "C"
