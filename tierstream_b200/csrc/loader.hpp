// The open's fill as a pipeline: reader threads read the units from their files while the opening thread copies what
// they read to the device, so the file reads, the host link and the readers of pinned units all run at once (the
// reference's startup loader, src/dg_load.hpp:84-95 and src/dg_ctx.cpp:1953-2016, does the same job).
//
// A unit with a slot lands on the device through a ring of caller-owned host buffers: consecutive slot units are
// packed into batches of buffer_bytes / stride units (at least one), a reader reads a whole batch into a free buffer,
// and the opening thread hands the batch to `submit` (which enqueues its copies and marks the buffer busy) and later
// to `recycle` (which waits until those copies are done) before the buffer is read into again. A unit without a slot
// is read in place into its host destination. Readers take batches first and pinned units while no buffer is free,
// and wait for a buffer only when no pinned unit is left. `submit` and `recycle` run on the calling thread only, so a
// CUDA stream and its events need no other thread; `read` runs on the reader threads.
#pragma once

#include <cstdint>
#include <functional>
#include <vector>

namespace tsb {

struct LoadUnit {
  int layer = 0, unit = 0;
  int32_t slot = -1;     // >= 0: to this device slot through the ring
  char* host = nullptr;  // slot < 0: read here in place
};

struct LoadCopy {
  int32_t slot;
  const char* data;  // the unit's bytes in a ring buffer
  size_t index;      // the unit's index in the loader's list
};

struct LoadStats {
  uint64_t slot_units = 0, host_units = 0, batches = 0;
  uint64_t recycles = 0;          // buffers waited for by the opening thread because a reader wanted one
  uint64_t reader_waits = 0;      // times a reader waited for a free buffer
  uint64_t max_in_flight = 0;     // batches submitted and not yet recycled, at most
  double seconds = 0, slot_seconds = 0;  // the whole run; up to the last batch submitted
};

// Reads every unit (read(unit, dst) reads its bytes to dst and checks them; it throws on failure) and submits every
// slot unit's batch; returns once every reader ended and every submitted buffer was recycled. The first failure of a
// reader, of submit or of recycle stops the readers and is rethrown after that. buffers may be empty only when no unit
// has a slot; stride >= the unit's bytes is each unit's offset step in a buffer (buffer_bytes >= stride).
LoadStats run_load(const std::vector<LoadUnit>& units, const std::vector<char*>& buffers, uint64_t buffer_bytes,
                   uint64_t stride, unsigned readers, const std::function<void(const LoadUnit&, char*)>& read,
                   const std::function<void(size_t, const std::vector<LoadCopy>&)>& submit,
                   const std::function<void(size_t)>& recycle);

}  // namespace tsb
