// The peer tier's planner and stores (peer.hpp).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <memory>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>

#include "ctx.hpp"
#include "errors.hpp"
#include "kernels.hpp"
#include "loader.hpp"
#include "peer.hpp"
#include "source_file.hpp"

namespace tsb {
namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    fail(SS_E_BACKEND, std::string(what) + ": " + cudaGetErrorString(e));
  }
}

// K3 over n units of unit_bytes each, unit i at at[i] (this device's memory), against want[i], in launches of up to
// 4096 units on `s`; returns the mismatches. Synchronous.
uint32_t hash_check(const std::vector<const uint8_t*>& at, const std::vector<uint64_t>& want, uint64_t unit_bytes,
                    cudaStream_t s) {
  constexpr size_t kChunk = 4096;
  const size_t nb = std::min(kChunk, at.size());
  if (!nb) return 0;
  void* buf = nullptr;
  ck(cudaMalloc(&buf, nb * (sizeof(dev::HashUnit) + 16) + 16), "cudaMalloc (store check)");
  auto* du = static_cast<dev::HashUnit*>(buf);
  auto* de = reinterpret_cast<uint64_t*>(du + nb);
  auto* dout = de + nb;
  auto* dmis = reinterpret_cast<uint32_t*>(dout + nb);  // [0] mismatches, [1] this check's staging timeouts
  uint32_t words[2] = {0, 0};
  try {
    ck(cudaMemsetAsync(dmis, 0, 8, s), "store check clear");
    for (size_t first = 0; first < at.size(); first += kChunk) {
      const size_t n = std::min(kChunk, at.size() - first);
      std::vector<dev::HashUnit> hu(n);
      for (size_t i = 0; i < n; ++i) {
        hu[i] = dev::HashUnit{};
        hu[i].n_spans = 1;
        hu[i].span[0] = at[first + i];
        hu[i].bytes[0] = unit_bytes;
      }
      ck(cudaMemcpyAsync(du, hu.data(), n * sizeof(dev::HashUnit), cudaMemcpyHostToDevice, s), "store check upload");
      ck(cudaMemcpyAsync(de, want.data() + first, n * 8, cudaMemcpyHostToDevice, s), "store check upload");
      ck(cudaError_t(dev::launch_xxh64(du, uint32_t(n), de, dout, nullptr, dmis, s, dmis + 1)), "xxh64 kernel");
      ck(cudaStreamSynchronize(s), "store check");  // the host tables are reused
    }
    ck(cudaMemcpy(words, dmis, 8, cudaMemcpyDeviceToHost), "store check result");
  } catch (...) {
    cudaFree(buf);
    throw;
  }
  cudaFree(buf);
  require(!words[1], SS_E_BACKEND, "peer tier: a staging copy of the xxh64 kernel did not complete");
  return words[0];
}

// [lo, lo + n) of unit `unit` of layer l read from the sources into dst (parts back to back in descriptor order).
void read_unit_range(const Layer& l, int unit, uint64_t lo, uint64_t n,
                     const std::vector<std::unique_ptr<SourceFile>>& files, char* dst) {
  uint64_t off = 0;
  for (const Part& p : l.parts) {
    const uint64_t a = std::max(lo, off), b = std::min(lo + n, off + p.bytes);
    if (a < b) files[size_t(p.source)]->read(dst + (a - lo), p.offset + uint64_t(unit) * p.stride + (a - off), b - a);
    off += p.bytes;
  }
}

}  // namespace

uint64_t stripe_bytes(uint64_t unit_bytes, uint32_t world) {
  require(world >= 1, SS_E_INVALID, "peer tier: world must be >= 1");
  const uint64_t s = (unit_bytes + world - 1) / world;
  return (s + 255) / 256 * 256;
}

std::vector<int64_t> striped_index(const std::vector<int32_t>& owner, uint64_t* owned) {
  std::vector<int64_t> index(owner.size(), -1);
  int64_t n = 0;
  for (size_t k = 0; k < owner.size(); ++k)
    if (owner[k] >= 0) index[k] = n++;
  if (owned) *owned = uint64_t(n);
  return index;
}

GatedKeys gated_keys(const Desc& d) {
  GatedKeys g;
  g.base.push_back(0);
  uint64_t keys = 0;
  for (size_t L = 0; L < d.layers.size(); ++L) {
    const Layer& l = d.layers[L];
    if (l.n_units == 0) continue;
    require(l.streamable, SS_E_UNSUPPORTED,
            "peer tier: layer " + std::to_string(l.index) + " has non-streamable units (every unit is gated)");
    if (!g.unit_bytes) g.unit_bytes = l.unit_bytes;
    require(l.unit_bytes == g.unit_bytes, SS_E_UNSUPPORTED, "peer tier: gated layers of different unit sizes");
    g.layers.push_back(int(L));
    keys += uint64_t(l.n_units);
    require(keys < 0x7fffffffull, SS_E_INVALID, "peer tier: more than 2^31 - 1 gated units");
    g.base.push_back(uint32_t(keys));
  }
  require(!g.layers.empty(), SS_E_INVALID, "peer tier: the descriptor has no streamable units");
  return g;
}

std::vector<int32_t> plan_owners(const uint64_t* counts, uint32_t keys, uint32_t world, const uint64_t* cap_units) {
  require(world >= 1 && world <= 1024, SS_E_INVALID, "tsb_peer_plan: world must be 1..1024");
  require(counts != nullptr || keys == 0, SS_E_INVALID, "tsb_peer_plan: null counts");
  std::vector<uint32_t> order(keys);
  std::iota(order.begin(), order.end(), 0u);
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return counts[a] > counts[b]; });
  std::vector<uint64_t> load(world, 0), units(world, 0);
  std::vector<int32_t> owner(keys, -1);
  for (uint32_t k : order) {
    int32_t best = -1;
    for (uint32_t r = 0; r < world; ++r) {
      if (cap_units && units[r] >= cap_units[r]) continue;
      if (best < 0 || load[r] < load[size_t(best)] ||
          (load[r] == load[size_t(best)] && units[r] < units[size_t(best)]))
        best = int32_t(r);
    }
    if (best < 0) continue;
    owner[k] = best;
    load[size_t(best)] += counts[k];
    ++units[size_t(best)];
  }
  return owner;
}

std::vector<int64_t> store_index(const std::vector<int32_t>& owner, uint32_t world, std::vector<uint64_t>* per_rank) {
  std::vector<uint64_t> n(world, 0);
  std::vector<int64_t> index(owner.size(), -1);
  for (size_t k = 0; k < owner.size(); ++k) {
    const int32_t o = owner[k];
    if (o < 0) continue;
    require(uint32_t(o) < world, SS_E_INVALID, "peer tier: owner " + std::to_string(o) + " of key " +
                                                   std::to_string(k) + " is not a rank below the world size");
    index[k] = int64_t(n[size_t(o)]++);
  }
  if (per_rank) *per_rank = n;
  return index;
}

PeerStore::PeerStore(const Desc& d, const std::vector<int32_t>& owner, int32_t rank, int device, bool verify, bool fill,
                     uint32_t layout, uint32_t world)
    : layout_(layout), device_(device) {
  const auto t0 = std::chrono::steady_clock::now();
  const GatedKeys gk = gated_keys(d);
  require(owner.size() == gk.keys(), SS_E_INVALID,
          "peer tier: the owner map has " + std::to_string(owner.size()) + " keys, the descriptor " +
              std::to_string(gk.keys()));
  require(rank >= 0, SS_E_INVALID, "peer tier: negative rank");
  require(layout == kWholeUnits || layout == kStriped, SS_E_INVALID,
          "peer tier: layout must be 0 (whole units) or 1 (striped)");
  const bool striped = layout == kStriped;
  require(!striped || (world >= 1 && world <= 1024 && uint32_t(rank) < world), SS_E_INVALID,
          "peer tier: a striped store needs world in 1..1024 and rank below it");
  require(!(striped && verify), SS_E_INVALID,
          "peer tier: a stripe cannot be checked against its unit's hash alone (check the tier once mapped)");
  DeviceScope on(device);  // the caller's current device comes back on return
  std::vector<std::pair<uint32_t, uint32_t>> mine;  // (gated ordinal, unit), key order
  for (uint32_t g = 0; g + 1 < gk.base.size(); ++g)
    for (uint32_t u = 0; u < gk.base[g + 1] - gk.base[g]; ++u) {
      const int32_t o = owner[gk.base[g] + u];
      if (striped ? o >= 0 : o == rank) mine.push_back({g, u});
    }
  // each unit's bytes held here: the whole unit, or this rank's stripe; slot i of the store at base + i * store_stride
  const uint64_t store_stride = striped ? stripe_bytes(gk.unit_bytes, world) : gk.unit_bytes;
  const uint64_t held_lo = striped ? uint64_t(rank) * store_stride : 0;
  const uint64_t held = striped ? stripe_len(gk.unit_bytes, store_stride, uint32_t(rank)) : gk.unit_bytes;
  units_ = mine.size();
  bytes_ = held ? units_ * store_stride : 0;
  unit_bytes_ = gk.unit_bytes;
  rank_ = rank;
  owner_ = owner;
  if (!bytes_) return;
  ck(cudaMalloc(reinterpret_cast<void**>(&base_), size_t(bytes_)), "cudaMalloc (peer store)");
  if (!fill) {
    fill_s_ = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return;
  }
  try {
    std::vector<std::unique_ptr<SourceFile>> files;
    for (const Source& s : d.sources) files.push_back(std::make_unique<SourceFile>(s.path, s.align, false));
    // the owned units (or stripes) through the open's fill pipeline (loader.hpp): reader threads read them into a
    // ring of pinned buffers (4 of up to 64 MiB), and this thread copies each full buffer into the store on one stream
    const uint64_t stride = (held + 4095) / 4096 * 4096;
    const uint64_t per = std::max<uint64_t>(1, std::min<uint64_t>((uint64_t(64) << 20) / stride, units_));
    const size_t nbuf = size_t(std::min<uint64_t>(4, (units_ + per - 1) / per));
    std::vector<char*> stage;
    std::vector<cudaEvent_t> ev;
    cudaStream_t s = nullptr;
    auto release = [&] {
      if (s) (void)cudaStreamSynchronize(s);  // (an error path: no copy may read a buffer being freed)
      for (char* p : stage) cudaFreeHost(p);
      for (cudaEvent_t e : ev) cudaEventDestroy(e);
      if (s) cudaStreamDestroy(s);
    };
    try {
      ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate (peer store)");
      for (size_t b = 0; b < nbuf; ++b) {
        char* p = nullptr;
        ck(cudaHostAlloc(reinterpret_cast<void**>(&p), size_t(per * stride), cudaHostAllocPortable),
           "cudaHostAlloc (peer store staging)");
        stage.push_back(p);
        cudaEvent_t e = nullptr;
        ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate (peer store)");
        ev.push_back(e);
      }
      std::vector<LoadUnit> units(mine.size());
      for (size_t i = 0; i < mine.size(); ++i)
        units[i] = LoadUnit{gk.layers[mine[i].first], int(mine[i].second), int32_t(i), nullptr};  // slot = store index
      const unsigned readers = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
      run_load(
          units, stage, per * stride, stride, readers,
          [&](const LoadUnit& lu, char* dst) {
            read_unit_range(d.layers[size_t(lu.layer)], lu.unit, held_lo, held, files, dst);
          },
          [&](size_t b, const std::vector<LoadCopy>& copies) {
            for (const LoadCopy& c : copies)
              ck(cudaMemcpyAsync(base_ + uint64_t(c.slot) * store_stride, c.data, size_t(held), cudaMemcpyHostToDevice,
                                 s),
                 "cudaMemcpyAsync (peer store fill)");
            ck(cudaEventRecord(ev[b], s), "cudaEventRecord (peer store fill)");
          },
          [&](size_t b) { ck(cudaEventSynchronize(ev[b]), "cudaEventSynchronize (peer store fill)"); });
      ck(cudaStreamSynchronize(s), "cudaStreamSynchronize (peer store fill)");
      // the store against the descriptor's hashes: K3 over every unit
      const bool hashes = !d.layers[size_t(gk.layers[0])].hash.empty();
      if (verify && hashes) {
        std::vector<const uint8_t*> at(mine.size());
        std::vector<uint64_t> want(mine.size());
        for (size_t i = 0; i < mine.size(); ++i) {
          at[i] = reinterpret_cast<const uint8_t*>(base_ + i * gk.unit_bytes);
          want[i] = d.layers[size_t(gk.layers[mine[i].first])].hash[mine[i].second];
        }
        const uint32_t mism = hash_check(at, want, gk.unit_bytes, s);
        require(mism == 0, SS_E_HASH,
                "peer tier: " + std::to_string(mism) + " stored unit(s) differ from their descriptor hashes");
      }
    } catch (...) {
      release();
      throw;
    }
    release();
  } catch (...) {
    cudaFree(base_);
    base_ = nullptr;
    throw;
  }
  fill_s_ = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

void ipc_export(const void* base, void* handle) {
  require(base && handle, SS_E_INVALID, "tsb_peer_store_export: an empty store has no handle");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "a CUDA IPC handle is 64 bytes");
  cudaIpcMemHandle_t h;
  ck(cudaIpcGetMemHandle(&h, const_cast<void*>(base)), "cudaIpcGetMemHandle (peer store)");
  std::memcpy(handle, &h, sizeof h);
}

void* ipc_map(const void* handle, int device) {
  require(handle != nullptr, SS_E_INVALID, "tsb_peer_map: null handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  int cur = 0;
  ck(cudaGetDevice(&cur), "cudaGetDevice");
  ck(cudaSetDevice(device), "cudaSetDevice (peer map)");
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  cudaSetDevice(cur);
  ck(e, "cudaIpcOpenMemHandle (peer store)");
  return p;
}

void ipc_unmap(void* base) {
  if (base) ck(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle (peer store)");
}

Migration migrate_store(PeerStore& dst, const std::vector<int32_t>& old_owner, const std::vector<char*>& old_base,
                        void* stream) {
  const auto t0 = std::chrono::steady_clock::now();
  const std::vector<int32_t>& now = dst.owner();
  require(dst.layout() == kWholeUnits, SS_E_UNSUPPORTED,
          "tsb_peer_store_migrate: a striped store does not depend on the owners (every rank holds a stripe of every "
          "owned unit), so a re-plan that keeps the owned units keeps the stores");
  require(old_owner.size() == now.size(), SS_E_INVALID,
          "tsb_peer_store_migrate: the old owner map has " + std::to_string(old_owner.size()) + " keys, the store's " +
              std::to_string(now.size()));
  const uint32_t world = uint32_t(old_base.size());
  std::vector<uint64_t> per;
  const std::vector<int64_t> old_index = store_index(old_owner, world, &per);
  Migration m;
  const uint64_t ub = dst.unit_bytes();
  DeviceScope on(dst.device());
  auto b = std::make_unique<dev::Batch>();
  uint64_t chunks = 0;
  auto launch = [&] {
    if (!b->n_copies) return;
    const int grid = int(std::min<uint64_t>(std::max<uint64_t>(chunks, 1), 296));
    ck(cudaError_t(dev::launch_batch(*b, grid, stream)), "land kernel (migration)");
    b->n_copies = 0;
    chunks = 0;
  };
  uint64_t i = 0;
  for (size_t k = 0; k < now.size(); ++k) {
    if (now[k] != dst.rank()) continue;
    const int32_t o = old_owner[k];
    require(o >= 0, SS_E_INVALID,
            "tsb_peer_store_migrate: key " + std::to_string(k) + " joins the tier (unowned before): a new store reads "
            "such units from their file (tsb_peer_store_create)");
    require(uint32_t(o) < world && old_base[size_t(o)], SS_E_INVALID,
            "tsb_peer_store_migrate: no store address for rank " + std::to_string(o));
    if (b->n_copies == dev::kMaxCopies) launch();
    b->copies[b->n_copies++] = {old_base[size_t(o)] + uint64_t(old_index[k]) * ub, dst.base() + i * ub, ub};
    chunks += (ub + (64u << 10) - 1) >> 16;
    ++m.units;
    if (o != dst.rank()) ++m.peer_units;
    ++i;
  }
  launch();
  ck(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "cudaStreamSynchronize (migration)");
  m.bytes = m.units * ub;
  m.seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  return m;
}

uint64_t verify_tier(const Desc& d, const PeerTier& t, int device) {
  const GatedKeys gk = gated_keys(d);
  require(t.owner.size() == gk.keys(), SS_E_INVALID, "tsb_peer_tier_verify: the tier covers other keys");
  require(!d.layers[size_t(gk.layers[0])].hash.empty(), SS_E_INVALID,
          "tsb_peer_tier_verify: the descriptor has no unit hashes");
  std::vector<uint32_t> keys;  // this rank's share, key order
  uint64_t pos = 0;
  for (uint32_t k = 0; k < gk.keys(); ++k)
    if (t.owned(k) && pos++ % t.world == uint32_t(t.rank)) keys.push_back(k);
  if (keys.empty()) return 0;
  const uint64_t ub = gk.unit_bytes;
  const size_t batch = size_t(std::max<uint64_t>(1, std::min<uint64_t>(keys.size(), (uint64_t(2) << 30) / ub)));
  DeviceScope on(device);
  char* scratch = nullptr;
  cudaStream_t s = nullptr;
  uint64_t mism = 0;
  try {
    ck(cudaMalloc(reinterpret_cast<void**>(&scratch), size_t(batch * ub)), "cudaMalloc (tier check)");
    ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate (tier check)");
    for (size_t first = 0; first < keys.size(); first += batch) {
      const size_t n = std::min(batch, keys.size() - first);
      std::vector<const uint8_t*> at(n);
      std::vector<uint64_t> want(n);
      for (size_t j = 0; j < n; ++j) {
        const uint32_t k = keys[first + j];
        char* dst = scratch + j * ub;
        t.pieces(k, ub, [&](const char* src, uint64_t off, uint64_t bytes, int32_t) {
          ck(cudaMemcpyAsync(dst + off, src, size_t(bytes), cudaMemcpyDefault, s), "cudaMemcpyAsync (tier check)");
        });
        const uint32_t g = uint32_t(std::upper_bound(gk.base.begin(), gk.base.end(), k) - gk.base.begin()) - 1;
        at[j] = reinterpret_cast<const uint8_t*>(dst);
        want[j] = d.layers[size_t(gk.layers[g])].hash[k - gk.base[g]];
      }
      mism += hash_check(at, want, ub, s);  // (stream-ordered after the gathers)
    }
  } catch (...) {
    if (s) {
      (void)cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
    cudaFree(scratch);
    throw;
  }
  cudaStreamDestroy(s);
  cudaFree(scratch);
  require(mism == 0, SS_E_HASH,
          "peer tier: " + std::to_string(mism) + " unit(s) gathered from the stores differ from their descriptor hashes");
  return keys.size();
}

PeerStore::~PeerStore() {
  if (base_) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device_);
    cudaFree(base_);
    cudaSetDevice(cur);
  }
}

}  // namespace tsb
