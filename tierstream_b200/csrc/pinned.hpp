// Mapped pinned host memory in large chunks. Anonymous mappings with transparent huge pages, populated by a pool of
// threads and then registered with CUDA (mapped, portable): on B200 boxes this pins 16 GiB in 0.6 s where
// cudaHostAlloc takes 6.7 s (the driver zeroes and pins 4 KiB pages one thread at a time). A chunk the system refuses
// that way comes from cudaHostAlloc instead.
#pragma once

#include <cstddef>
#include <vector>

namespace tsb {

struct PinnedChunk {
  void* ptr = nullptr;
  size_t bytes = 0;
  bool registered = false;  // mmap + cudaHostRegister (else cudaHostAlloc)
};

// Chunks of the given sizes on `device` (mapped into its address space, usable by kernels at the same address);
// throws SS_E_NOMEM when the memory cannot be had either way.
std::vector<PinnedChunk> alloc_pinned(const std::vector<size_t>& sizes, int device);
void free_pinned(std::vector<PinnedChunk>& chunks) noexcept;

}  // namespace tsb
