// The tsb_* entry points of include/tierstream/tsb.h.
#include <cuda_runtime.h>

#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <thread>
#include <string>
#include <vector>

#include "dg_core.hpp"
#include "errors.hpp"
#include "kernels.hpp"
#include "loader.hpp"
#include "read_ahead.hpp"
#include "source_file.hpp"
#include "tierstream/tsb.h"
#include "xxh64.hpp"

namespace tsb {
void dg_replay(const tsb_dg_replay_config* c, const int32_t* ids, const int32_t* preds, int32_t* tables,
               uint64_t* stats, const uint8_t* src_units, uint64_t* read_sum);
void dg_async_replay(const tsb_dg_replay_config* c, const int32_t* ids, const int32_t* preds,
                     const uint8_t* src_units, uint32_t seed, uint32_t delay_us, int32_t mutation, uint64_t* read_sum,
                     uint64_t* races);
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

ss_status tsb_test_dg_async_replay(const tsb_dg_replay_config* cfg, const int32_t* ids, const int32_t* preds,
                                   const uint8_t* src_units, uint32_t seed, uint32_t delay_us, int32_t mutation,
                                   uint64_t* read_sum, uint64_t* races) {
  return run([&] { tsb::dg_async_replay(cfg, ids, preds, src_units, seed, delay_us, mutation, read_sum, races); });
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
    tsb::AsyncReads q(threads, [&](uint32_t i, char* out, unsigned) { f.read(out, offsets[i], bytes); });
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

ss_status tsb_test_read_ahead(const char* path, const uint64_t* offsets, uint32_t n_units, uint64_t unit_bytes,
                              uint32_t buffers, uint32_t threads, uint32_t read_delay_us, const int32_t* script,
                              uint32_t n_ops, uint64_t* sums, int32_t* codes, uint64_t* stats) {
  return run([&] {
    tsb::require(path && (offsets || !n_units) && (script || !n_ops) && unit_bytes >= 1 && buffers <= 64 &&
                     threads >= 1 && threads <= 64,
                 SS_E_INVALID, "tsb_test_read_ahead: bad argument");
    tsb::SourceFile f(path, 4096, false);
    const uint64_t stride = (unit_bytes + 4095) / 4096 * 4096;
    std::vector<char*> bufs;
    struct Free {
      std::vector<char*>* b;
      ~Free() {
        for (char* p : *b) std::free(p);
      }
    } guard{&bufs};
    for (uint32_t i = 0; i < buffers; ++i) {
      bufs.push_back(static_cast<char*>(std::aligned_alloc(4096, size_t(stride))));
      tsb::require(bufs.back() != nullptr, SS_E_NOMEM, "tsb_test_read_ahead: buffer");
    }
    tsb::ReadAhead ra(bufs, threads, [&](int, int unit, char* dst) {
      if (read_delay_us) std::this_thread::sleep_for(std::chrono::microseconds(read_delay_us));
      tsb::require(unit >= 0 && uint32_t(unit) < n_units, SS_E_INVALID, "tsb_test_read_ahead: unit");
      f.read(dst, offsets[unit], unit_bytes);
      return unit_bytes;
    });
    uint32_t claims = 0, ends = 0;
    for (uint32_t i = 0; i < n_ops; ++i) {
      const int32_t op = script[3 * i], unit = script[3 * i + 1], arg = script[3 * i + 2];
      if (op == 0) {
        ra.request(0, unit);
      } else if (op == 1) {  // a fetch: its claim, the read's end, its copy (arg 0 ends well, 1 fails before, 2 after)
        uint64_t s = 0;
        int32_t code = 0;
        if (auto e = ra.claim(0, unit)) {
          ss_status st = SS_OK;
          std::string msg;
          if (const char* b = ra.wait(*e, &st, &msg)) {
            for (uint64_t k = 0; k < unit_bytes; ++k) s += uint64_t(uint8_t(b[k])) * (k % 251 + 1);
            code = 1;
            ra.done(*e, arg == 0, arg == 2);
          } else {
            code = -int32_t(st);
          }
        }
        if (sums) sums[claims] = s;
        if (codes) codes[claims] = code;
        ++claims;
      } else if (op == 2) {
        const tsb::RaStats f = ra.end_forward();
        const uint64_t v[7] = {f.requested, f.read, f.landed, f.unused, f.failed, ra.totals().fallback, f.bytes};
        if (stats) std::memcpy(stats + 7 * size_t(ends), v, sizeof v);
        ++ends;
      } else if (op == 3) {
        std::this_thread::sleep_for(std::chrono::microseconds(std::max(0, arg)));
      } else {
        tsb::fail(SS_E_INVALID, "tsb_test_read_ahead: unknown op");
      }
    }
  });
}

ss_status tsb_test_load(const char* path, const uint64_t* offsets, const int32_t* targets, uint32_t n,
                        uint64_t unit_bytes, void* device, void* host, uint32_t buffers, uint64_t buffer_bytes,
                        uint32_t readers, int direct, uint32_t copy_delay_us, int32_t fail_batch, uint64_t* stats) {
  return run([&] {
    tsb::require(path && (offsets || !n) && (targets || !n) && unit_bytes >= 1 && readers >= 1 && readers <= 64 &&
                     buffers <= 64,
                 SS_E_INVALID, "tsb_test_load: bad argument");
    const uint64_t stride = (unit_bytes + 4095) / 4096 * 4096;
    tsb::SourceFile f(path, 4096, direct != 0);
    std::vector<tsb::LoadUnit> units(n);
    for (uint32_t i = 0; i < n; ++i) {
      units[i].unit = int(i);
      units[i].slot = targets[i];
      if (targets[i] < 0) {
        tsb::require(host != nullptr, SS_E_INVALID, "tsb_test_load: a host unit and no host area");
        units[i].host = static_cast<char*>(host) + uint64_t(-int64_t(targets[i]) - 1) * stride;
      } else {
        tsb::require(device != nullptr, SS_E_INVALID, "tsb_test_load: a slot unit and no device area");
      }
    }
    struct Ring {
      std::vector<char*> p;
      ~Ring() {
        for (char* b : p) std::free(b);
      }
    } ring;
    for (uint32_t b = 0; b < buffers; ++b) {
      ring.p.push_back(static_cast<char*>(std::aligned_alloc(4096, size_t((buffer_bytes + 4095) / 4096 * 4096))));
      tsb::require(ring.p.back() != nullptr, SS_E_NOMEM, "tsb_test_load: ring buffer");
    }
    // a copy engine of its own: copies run in submission order on one thread, copy_delay_us after they were submitted,
    // and a buffer's event completes when its last copy did
    std::mutex mu;
    std::condition_variable cv;
    std::deque<std::pair<uint64_t, std::vector<tsb::LoadCopy>>> q;
    std::vector<uint64_t> event(buffers, 0);
    uint64_t seq = 0, completed = 0, batch = 0;
    bool stop = false;
    std::thread engine([&] {
      std::unique_lock<std::mutex> lk(mu);
      for (;;) {
        cv.wait(lk, [&] { return stop || !q.empty(); });
        if (q.empty()) return;
        auto job = std::move(q.front());
        q.pop_front();
        lk.unlock();
        if (copy_delay_us) std::this_thread::sleep_for(std::chrono::microseconds(copy_delay_us));
        for (const tsb::LoadCopy& c : job.second)
          std::memcpy(static_cast<char*>(device) + uint64_t(c.slot) * stride, c.data, size_t(unit_bytes));
        lk.lock();
        completed = job.first;
        cv.notify_all();
      }
    });
    tsb::LoadStats st;
    std::exception_ptr err;
    try {
      st = tsb::run_load(
          units, ring.p, buffer_bytes, stride, readers,
          [&](const tsb::LoadUnit& u, char* dst) { f.read(dst, offsets[u.unit], unit_bytes); },
          [&](size_t buf, const std::vector<tsb::LoadCopy>& copies) {
            std::lock_guard<std::mutex> lk(mu);
            tsb::require(int32_t(batch++) != fail_batch, SS_E_BACKEND, "tsb_test_load: the copy engine refused");
            q.emplace_back(++seq, copies);
            event[buf] = seq;
            cv.notify_all();
          },
          [&](size_t buf) {
            std::unique_lock<std::mutex> lk(mu);
            cv.wait(lk, [&] { return completed >= event[buf]; });
          });
    } catch (...) {
      err = std::current_exception();
    }
    {
      std::lock_guard<std::mutex> lk(mu);
      stop = true;
      cv.notify_all();
    }
    engine.join();
    if (err) std::rethrow_exception(err);
    if (stats) {
      const uint64_t v[6] = {st.slot_units, st.host_units, st.batches, st.recycles, st.reader_waits, st.max_in_flight};
      std::memcpy(stats, v, sizeof v);
    }
  });
}

uint64_t tsb_xxh64(const void* data, size_t len, uint64_t seed) { return tsb::xxh64(data, len, seed); }

int tsb_cuda_arch(void) { return 100; }

}  // extern "C"
