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

}  // namespace

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

PeerStore::PeerStore(const Desc& d, const std::vector<int32_t>& owner, int32_t rank, int device, bool verify, bool fill)
    : device_(device) {
  const auto t0 = std::chrono::steady_clock::now();
  const GatedKeys gk = gated_keys(d);
  require(owner.size() == gk.keys(), SS_E_INVALID,
          "peer tier: the owner map has " + std::to_string(owner.size()) + " keys, the descriptor " +
              std::to_string(gk.keys()));
  require(rank >= 0, SS_E_INVALID, "peer tier: negative rank");
  DeviceScope on(device);  // the caller's current device comes back on return
  std::vector<std::pair<uint32_t, uint32_t>> mine;  // (gated ordinal, unit), key order
  for (uint32_t g = 0; g + 1 < gk.base.size(); ++g)
    for (uint32_t u = 0; u < gk.base[g + 1] - gk.base[g]; ++u)
      if (owner[gk.base[g] + u] == rank) mine.push_back({g, u});
  units_ = mine.size();
  bytes_ = units_ * gk.unit_bytes;
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
    // the owned units through the open's fill pipeline (loader.hpp): reader threads read them into a ring of pinned
    // buffers (4 of up to 64 MiB), and this thread copies each full buffer into the store on one stream
    const uint64_t stride = (gk.unit_bytes + 4095) / 4096 * 4096;
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
            const Layer& l = d.layers[size_t(lu.layer)];
            uint64_t off = 0;
            for (const Part& p : l.parts) {
              files[size_t(p.source)]->read(dst + off, p.offset + uint64_t(lu.unit) * p.stride, p.bytes);
              off += p.bytes;
            }
          },
          [&](size_t b, const std::vector<LoadCopy>& copies) {
            for (const LoadCopy& c : copies)
              ck(cudaMemcpyAsync(base_ + uint64_t(c.slot) * gk.unit_bytes, c.data, size_t(gk.unit_bytes),
                                 cudaMemcpyHostToDevice, s),
                 "cudaMemcpyAsync (peer store fill)");
            ck(cudaEventRecord(ev[b], s), "cudaEventRecord (peer store fill)");
          },
          [&](size_t b) { ck(cudaEventSynchronize(ev[b]), "cudaEventSynchronize (peer store fill)"); });
      ck(cudaStreamSynchronize(s), "cudaStreamSynchronize (peer store fill)");
      // the store against the descriptor's hashes: K3 over every unit, in launches of up to 4096 units
      const bool hashes = !d.layers[size_t(gk.layers[0])].hash.empty();
      if (verify && hashes) {
        const size_t chunk = 4096;
        void* buf = nullptr;
        const size_t nb = std::min<size_t>(chunk, units_);
        ck(cudaMalloc(&buf, nb * (sizeof(dev::HashUnit) + 16) + 16), "cudaMalloc (peer store verify)");
        auto* du = static_cast<dev::HashUnit*>(buf);
        auto* de = reinterpret_cast<uint64_t*>(du + nb);
        auto* dout = de + nb;
        auto* dmis = reinterpret_cast<uint32_t*>(dout + nb);  // [0] mismatches, [1] this fill's staging timeouts
        uint32_t words[2] = {0, 0};
        try {
          ck(cudaMemsetAsync(dmis, 0, 8, s), "peer store verify clear");
          for (size_t first = 0; first < units_; first += chunk) {
            const size_t n = std::min(chunk, size_t(units_) - first);
            std::vector<dev::HashUnit> hu(n);
            std::vector<uint64_t> want(n);
            for (size_t i = 0; i < n; ++i) {
              const auto [g, u] = mine[first + i];
              const Layer& l = d.layers[size_t(gk.layers[g])];
              hu[i] = dev::HashUnit{};
              hu[i].n_spans = 1;
              hu[i].span[0] = reinterpret_cast<const uint8_t*>(base_ + (first + i) * gk.unit_bytes);
              hu[i].bytes[0] = gk.unit_bytes;
              want[i] = l.hash[u];
            }
            ck(cudaMemcpyAsync(du, hu.data(), n * sizeof(dev::HashUnit), cudaMemcpyHostToDevice, s), "verify upload");
            ck(cudaMemcpyAsync(de, want.data(), n * 8, cudaMemcpyHostToDevice, s), "verify upload");
            ck(cudaError_t(dev::launch_xxh64(du, uint32_t(n), de, dout, nullptr, dmis, s, dmis + 1)), "xxh64 kernel");
            ck(cudaStreamSynchronize(s), "peer store verify");  // the host tables are reused
          }
          ck(cudaMemcpy(words, dmis, 8, cudaMemcpyDeviceToHost), "peer store verify result");
          require(!words[1], SS_E_BACKEND, "peer tier: a staging copy of the xxh64 kernel did not complete");
        } catch (...) {
          cudaFree(buf);
          throw;
        }
        cudaFree(buf);
        const uint32_t mism = words[0];
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
