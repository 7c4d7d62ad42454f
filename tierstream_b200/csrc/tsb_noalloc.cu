// tsb_xxh64_units_static: tsb_xxh64_units with its unit table in a file-scope device array instead of caller memory.
//
// The device xxh64 kernel reads a table of units (72 bytes each: up to four spans and their lengths). tsb_xxh64_units
// takes that table's device memory from the caller; this entry point keeps it in g_unit_table below, so a caller that
// cannot allocate device memory (an engine whose HBM the plan's arena already covers, or one whose allocator is not
// reachable from the thread doing the check) can still hash units on the device.
//
// Limits and rules:
// - at most kStaticUnits units per call; larger n is refused with SS_E_INVALID;
// - the first call on each device looks the table's address up (cudaGetSymbolAddress, which may load this module);
//   make that first call before any stream capture on the device;
// - nothing in the table has to start at zero: each call writes the n entries it uses before the kernel reads them.
//   The caller's *mismatches_dev is added to, not cleared, as with tsb_xxh64_units;
// - there is one table per device: calls that overlap on the same device (other host threads, or other streams before
//   this call's stream has finished) race on it. This call returns after its kernel finished, like tsb_xxh64_units.
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <vector>

#include "errors.hpp"
#include "kernels.hpp"
#include "tierstream/tsb.h"

namespace tsb {
const char* set_error(const std::string& msg);
}

namespace {

constexpr uint32_t kStaticUnits = TSB_XXH64_STATIC_MAX_UNITS;  // 4096 x 72 B = 288 KiB of device memory
constexpr int kMaxDevices = 64;

static __device__ __align__(256) tsb::dev::HashUnit g_unit_table[kStaticUnits];

std::mutex g_mu;
tsb::dev::HashUnit* g_table_ptr[kMaxDevices] = {};

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    tsb::fail(SS_E_BACKEND, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// The table's device address on the current device, looked up once per device.
tsb::dev::HashUnit* table_for_current_device() {
  int dev = -1;
  ck(cudaGetDevice(&dev), "tsb_xxh64_units_static: cudaGetDevice");
  tsb::require(dev >= 0 && dev < kMaxDevices, SS_E_BACKEND, "tsb_xxh64_units_static: device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_table_ptr[dev]) {
    void* p = nullptr;
    ck(cudaGetSymbolAddress(&p, g_unit_table), "tsb_xxh64_units_static: cudaGetSymbolAddress");
    tsb::require(p != nullptr, SS_E_BACKEND, "tsb_xxh64_units_static: no device address for the unit table");
    g_table_ptr[dev] = static_cast<tsb::dev::HashUnit*>(p);
  }
  return g_table_ptr[dev];
}

}  // namespace

extern "C" ss_status tsb_xxh64_units_static(const void* const* spans, const uint64_t* span_bytes,
                                            const uint32_t* n_spans, uint32_t n, const uint64_t* expect_dev,
                                            uint64_t* out_dev, uint32_t* mismatches_dev, void* stream) {
  try {
    if (!n) return SS_OK;
    tsb::require(n <= kStaticUnits, SS_E_INVALID,
                 "tsb_xxh64_units_static: at most " + std::to_string(kStaticUnits) + " units per call, got " +
                     std::to_string(n));
    tsb::require(spans && span_bytes && n_spans && out_dev, SS_E_INVALID, "tsb_xxh64_units_static: null argument");
    tsb::require(!expect_dev || mismatches_dev, SS_E_INVALID,
                 "tsb_xxh64_units_static: expected hashes need a mismatch word");
    std::vector<tsb::dev::HashUnit> u(n);
    for (uint32_t i = 0; i < n; ++i) {
      tsb::require(n_spans[i] >= 1 && n_spans[i] <= 4, SS_E_INVALID, "tsb_xxh64_units_static: 1..4 spans per unit");
      u[i] = tsb::dev::HashUnit{};
      u[i].n_spans = n_spans[i];
      for (uint32_t s = 0; s < n_spans[i]; ++s) {
        u[i].span[s] = static_cast<const uint8_t*>(spans[4 * size_t(i) + s]);
        u[i].bytes[s] = span_bytes[4 * size_t(i) + s];
      }
    }
    tsb::dev::HashUnit* table = table_for_current_device();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ck(cudaMemcpyAsync(table, u.data(), u.size() * sizeof(tsb::dev::HashUnit), cudaMemcpyHostToDevice, s),
       "tsb_xxh64_units_static: unit table upload");
    ck(cudaError_t(tsb::dev::launch_xxh64(table, n, expect_dev, out_dev, nullptr, mismatches_dev, s)), "xxh64 kernel");
    ck(cudaStreamSynchronize(s), "tsb_xxh64_units_static: sync");
    uint32_t timeouts = 0;
    ck(cudaError_t(tsb::dev::xxh64_take_timeouts(&timeouts)), "tsb_xxh64_units_static: timeout word");
    tsb::require(!timeouts, SS_E_BACKEND,
                 "tsb_xxh64_units_static: a staging copy of the xxh64 kernel did not complete");
    return SS_OK;
  } catch (const tsb::Error& e) {
    tsb::set_error(e.what());
    return e.status();
  } catch (const std::exception& e) {
    tsb::set_error(e.what());
    return SS_E_BACKEND;
  }
}
