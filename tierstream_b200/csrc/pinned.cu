// Mapped pinned host memory in large chunks (pinned.hpp).
#include <cuda_runtime.h>
#include <sys/mman.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>

#include "ctx.hpp"
#include "errors.hpp"
#include "pinned.hpp"

namespace tsb {

std::vector<PinnedChunk> alloc_pinned(const std::vector<size_t>& sizes, int device) {
  std::vector<PinnedChunk> out(sizes.size());
  for (size_t i = 0; i < sizes.size(); ++i) out[i].bytes = sizes[i];
  if (sizes.empty()) return out;
  DeviceScope on(device);
  // map and populate in parallel (page faults and zeroing spread over the threads)
  std::atomic<size_t> next{0};
  const size_t nth = std::min<size_t>(sizes.size(), std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
  std::vector<std::thread> th;
  for (size_t t = 0; t < nth; ++t)
    th.emplace_back([&] {
      for (size_t i; (i = next.fetch_add(1)) < out.size();) {
        void* m = mmap(nullptr, out[i].bytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
        if (m == MAP_FAILED) continue;
        (void)madvise(m, out[i].bytes, MADV_HUGEPAGE);  // best effort
        std::memset(m, 0, out[i].bytes);
        out[i].ptr = m;
      }
    });
  for (auto& t : th) t.join();
  std::string err;
  for (PinnedChunk& c : out) {
    if (c.ptr) {
      if (cudaHostRegister(c.ptr, c.bytes, cudaHostRegisterMapped | cudaHostRegisterPortable) == cudaSuccess) {
        c.registered = true;
        continue;
      }
      (void)cudaGetLastError();
      munmap(c.ptr, c.bytes);
      c.ptr = nullptr;
    }
    void* p = nullptr;  // the fallback
    const cudaError_t e = cudaHostAlloc(&p, c.bytes, cudaHostAllocMapped | cudaHostAllocPortable);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      err = std::string("cudaHostAlloc (pinned chunk): ") + cudaGetErrorString(e);
      break;
    }
    c.ptr = p;
  }
  if (!err.empty()) {
    free_pinned(out);
    fail(SS_E_NOMEM, err);
  }
  return out;
}

void free_pinned(std::vector<PinnedChunk>& chunks) noexcept {
  for (PinnedChunk& c : chunks) {
    if (!c.ptr) continue;
    if (c.registered) {
      cudaHostUnregister(c.ptr);
      munmap(c.ptr, c.bytes);
    } else {
      cudaFreeHost(c.ptr);
    }
    c.ptr = nullptr;
  }
  chunks.clear();
}

}  // namespace tsb
