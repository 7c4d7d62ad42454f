// The library's device kernels (kernels.cu, sm_100a) and their launchers. Every launcher only enqueues on the given
// stream (legal during stream capture), allocates nothing and returns the launch's cudaError_t as an int.
#pragma once

#include <cstdint>

namespace tsb {
namespace dev {

// ---- K1 / K5: batched copies (and K4, the same batch HBM -> HBM) ----
// One copy: `bytes` from src to dst; either side may be device memory, mapped pinned host memory or a peer GPU's
// memory (P2P). A batch's copies must not overlap each other.
struct Copy {
  const void* src;
  void* dst;
  uint64_t bytes;
};
// Entries published after every copy of the batch landed: slot_of[key] = val (release at system scope), then
// *ready_word = ready_val when ready_word is set. done_counter: one device word per stream the batches run on (the
// last block to finish publishes and rezeroes it).
constexpr uint32_t kMaxCopies = 384;
constexpr uint32_t kMaxEntries = 128;
struct Batch {
  uint32_t n_copies = 0, n_entries = 0;
  int32_t* slot_of = nullptr;
  uint32_t* ready_word = nullptr;
  uint32_t ready_val = 0;
  uint32_t* done_counter = nullptr;
  Copy copies[kMaxCopies];
  uint32_t entry_key[kMaxEntries];
  int32_t entry_val[kMaxEntries];
};
int launch_batch(const Batch& b, int blocks, void* stream);
// K4: the same batch, HBM -> HBM only, staged through shared memory by TMA bulk copies (one warp per CTA, 192 KiB of
// shared memory: one CTA per SM). Every copy 16-byte aligned with a 16-byte multiple size (move_fits), else
// cudaErrorInvalidValue. move_take_timeouts: load waits that ran out since the last call, then reset (synchronous).
bool move_fits(const Batch& b);
int launch_move(const Batch& b, int blocks, void* stream);
int move_take_timeouts(uint32_t* out);

// ---- K3: device xxh64 of whole units ----
// A unit is up to 4 spans hashed back to back (a gated unit's parts in the arena). out[i] = the hash; when expect is
// given, a mismatch increments *mismatches and sets bad[i] = 1 (bad may be null). timeouts_dev: the word counting
// staging waits that ran out (null: this library's per-device word, read by xxh64_take_timeouts); a failed unit is
// hashed as 0 and reported as a mismatch.
struct HashUnit {
  const uint8_t* span[4];
  uint64_t bytes[4];
  uint32_t n_spans;
  uint32_t pad;
};
int launch_xxh64(const HashUnit* units_dev, uint32_t n, const uint64_t* expect_dev, uint64_t* out_dev,
                 uint32_t* bad_dev, uint32_t* mismatches_dev, void* stream, uint32_t* timeouts_dev = nullptr);
// Staging waits of the xxh64 kernel that ran out since the last call on this device (launches given no timeout word),
// then reset; synchronous. Non-zero means the device did not complete a bulk copy in 2 s.
int xxh64_take_timeouts(uint32_t* out);
// K3 over landed slots of a device-gated arena (the landing check), passed by value in the launch: unit i is key[i]
// in slot[i] (part p at arena[p] + slot x part_bytes[p]), compared with expect[key]. A mismatch (or a unit whose
// staging wait ran out, counted in *timeouts) adds 1 to *bad_count, writes (key, slot) at bad_log[2 x its index] while
// the log has room (kBadLog entries), then *bad_flag = 1; bad_log and bad_flag are mapped host memory, written with
// system-scope stores so the host reads them without a device call. When every CTA of the launch finished, its last
// one resets *done_cnt and stores done_val to *done_word (mapped, release at system scope): the host learns of a
// finished launch without recording an event after it.
constexpr uint32_t kMaxVerify = 256, kBadLog = 64;
struct VerifyBatch {
  const uint8_t* arena[4];
  uint64_t part_bytes[4];
  uint32_t n_parts, n;
  const uint64_t* expect;  // [keys], device
  uint32_t* bad_count;     // device
  uint32_t* bad_log;       // mapped host, 2 x kBadLog words
  uint32_t* bad_flag;      // mapped host
  uint32_t* timeouts;      // device
  uint32_t* done_cnt;      // device, zero before the launch
  uint32_t* done_word;     // mapped host
  uint32_t done_val, pad;
  uint32_t key[kMaxVerify];
  int32_t slot[kMaxVerify];
};
int launch_xxh64_landed(const VerifyBatch& b, void* stream);

// ---- K2: device-gated decode control kernels ----
// The record an export writes for the service (mapped host memory); the layout is the reference's DgRecord
// (dg_proto.hpp:15-25): 288 bytes.
constexpr uint32_t kMaxIds = 64;
struct DgRecord {
  uint32_t n_ids, n_pred_promised, mask_lo, mask_hi;
  uint32_t seq, pad[3];
  uint32_t ids[kMaxIds];
};
struct DgPredRecord {
  uint32_t n_pred, pad[3];
  uint32_t pred[kMaxIds];
};
static_assert(sizeof(DgRecord) == 288 && sizeof(DgPredRecord) == 272, "record layout");
enum DgErr : uint32_t { kDgOk = 0, kDgTimeout = 1, kDgBadId = 2, kDgHostAbort = 3, kDgDesync = 4, kDgAbsent = 5 };
constexpr uint32_t kSkipWait = 1;  // test mutation: the wait kernel returns at once

// Every pointer the control kernels use, fixed at open (captured graphs replay for the context's life).
struct DgDev {
  // device memory
  uint32_t* seq;
  uint32_t* abort;
  uint32_t* err_count;
  uint32_t* err_code;
  uint32_t* err_aux;
  uint32_t* any_miss;    // [G]
  uint32_t* ready;       // [G], written after a layer's copies and entries
  uint32_t* absent_err;
  const int32_t* slot_of;
  const uint32_t* unit_base;  // [G + 1]
  // mapped host memory (device addresses)
  DgRecord* rec;
  DgPredRecord* prec;
  uint32_t* flag;
  uint32_t* pflag;
  uint32_t* done;
  uint32_t* m_err_code;
  uint32_t* m_err_aux;
  uint32_t* host_abort;
  uint32_t* host_seq;
  uint32_t* began;
  uint32_t* m_err_count;
  unsigned long long* stamps;  // diag: [4g] export, [4g + 1] wait entry, [4g + 2] ready seen; null = off
  unsigned long long timeout_ns;
  uint32_t test_flags;
};
int launch_dg_begin(const DgDev& d, void* stream);
int launch_dg_export(const DgDev& d, uint32_t g, const int32_t* ids, uint32_t n, uint32_t n_pred, void* stream);
int launch_dg_predict(const DgDev& d, uint32_t g, const int32_t* ids, uint32_t n, void* stream);
int launch_dg_wait(const DgDev& d, uint32_t g, void* stream);
int launch_dg_end(const DgDev& d, void* stream);
// Loads every kernel of this file (no lazy module load inside a capture).
int preload();

}  // namespace dev
}  // namespace tsb
