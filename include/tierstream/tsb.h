/* tierstream B200 runtime: entry points beyond the reference ABI (include/strix_stream/ss.h). Plain pointers and
 * sizes only. Device pointers are CUDA device addresses (or mapped pinned host addresses), streams are cudaStream_t
 * passed as void* (NULL = the legacy default stream). Every function returns an ss_status; the message of a failure is
 * in ss_last_error(). */
#ifndef TIERSTREAM_TSB_H
#define TIERSTREAM_TSB_H

#include "../strix_stream/ss.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- K1 / K5: batched copies (the land kernel) ----
 * n copies of bytes[i] bytes from src[i] to dst[i] in one launch (copies must not overlap each other; any side may be
 * device memory, mapped pinned host memory or a peer device's memory). Then, when n_entries > 0, slot_of[keys[j]] =
 * vals[j], and when ready_word is not NULL, *ready_word = ready_val, published once every copy landed. counter: one
 * zeroed device word owned by the caller's stream (used and re-zeroed by the launch; NULL when nothing is published).
 * At most 384 copies and 128 entries per call. Replaces, per miss, the reference's cudaMemcpyAsync per part plus a
 * cuStreamWriteValue32 per entry and ready word (dg_ctx.cpp:163-216). */
SS_API ss_status tsb_land(const void* const* src, void* const* dst, const uint64_t* bytes, uint32_t n,
                          int32_t* slot_of, const uint32_t* keys, const int32_t* vals, uint32_t n_entries,
                          uint32_t* ready_word, uint32_t ready_val, uint32_t* counter, uint32_t blocks, void* stream);

/* ---- K4: HBM -> HBM moves through shared memory (TMA bulk copies) ----
 * The same batch as tsb_land, every copy device memory to device memory with 16-byte aligned addresses and 16-byte
 * multiple sizes (else SS_E_INVALID): each 64 KiB chunk a bulk load into shared memory and a bulk store out, three
 * chunks in flight per CTA, one CTA per SM. What reset compaction (ss_dg_reset_open) runs. tsb_move_timeouts: the
 * chunk loads that did not complete within 2 s since the last call (their batch publishes nothing), then reset; -1 on
 * a device error. */
SS_API ss_status tsb_move(const void* const* src, void* const* dst, const uint64_t* bytes, uint32_t n,
                          int32_t* slot_of, const uint32_t* keys, const int32_t* vals, uint32_t n_entries,
                          uint32_t* ready_word, uint32_t ready_val, uint32_t* counter, uint32_t blocks, void* stream);
SS_API int tsb_move_timeouts(void);

/* ---- K3: device xxh64 of whole units ----
 * Unit i is n_spans[i] (1..4) spans spans[4 i + s] of span_bytes[4 i + s] bytes hashed back to back (a gated unit's
 * parts). units_dev: device scratch of n x 72 bytes (the unit table is staged there); out_dev: n hashes (device);
 * expect_dev (may be NULL): n expected hashes, mismatches counted into *mismatches_dev (device word, not cleared).
 * Bit-exact with the reference's host xxh64 (xxh64.cpp:39-112). Returns after the kernel finished; SS_E_BACKEND when a
 * staging copy inside the kernel did not complete in 2 s. That check reads and clears one word per device shared with
 * tsb_xxh64_units_static: a call that overlaps another on the same device may report the other's timeout (the
 * library's own verifications use words of their own). */
SS_API ss_status tsb_xxh64_units(const void* const* spans, const uint64_t* span_bytes, const uint32_t* n_spans,
                                 uint32_t n, void* units_dev, const uint64_t* expect_dev, uint64_t* out_dev,
                                 uint32_t* mismatches_dev, void* stream);

/* ---- K3 without caller scratch (no reference counterpart) ----
 * tsb_xxh64_units with the unit table in a device array of this library (TSB_XXH64_STATIC_MAX_UNITS units, 288 KiB)
 * instead of caller memory: for callers that cannot allocate device memory. n above the maximum returns SS_E_INVALID.
 * The first call on a device looks the array up (make it before any stream capture on that device). The table needs
 * no zeroing; *mismatches_dev is added to, not cleared. One table per device: overlapping calls on a device race.
 * Returns after the kernel finished; its timeout report shares a word with tsb_xxh64_units (above). */
#define TSB_XXH64_STATIC_MAX_UNITS 4096u
SS_API ss_status tsb_xxh64_units_static(const void* const* spans, const uint64_t* span_bytes, const uint32_t* n_spans,
                                        uint32_t n, const uint64_t* expect_dev, uint64_t* out_dev,
                                        uint32_t* mismatches_dev, void* stream);

/* ---- Deterministic replay of the device-gated slot cache on the host (test hook) ----
 * The same configuration and outputs as the reference harness's replay: this library's slot cache (dg_core.cpp)
 * driven in the service thread's order by a host mover whose events are complete when queried. tables: [tokens][keys]
 * slot_of after each boundary; stats: [tokens][16] (tokens, lookups, misses, covered, fetched, prefetched,
 * prefetch_used, resurrected, bank_serves, collected_mid, evicted, evict_short, writebacks_done, wb_deferred,
 * wb_cancelled, wb_forced); read_sum (optional, with move_bytes and src_units): per (token, g, id) the checksum
 * sum(byte * (pos % 251 + 1)) found through the table after the layer's demand. */
typedef struct tsb_dg_replay_config {
  uint32_t n_gated;
  const uint32_t* n_units;
  uint32_t n_parts;
  const uint64_t* part_bytes;
  uint32_t persistent_slots, bank_slots, blocks, spare_target;
  uint32_t prefetch_reserve; /* 0xFFFFFFFF = auto */
  uint32_t prefetch_per_layer, prefetch_per_token;
  uint32_t wb_defer, wb_on_d2h;
  uint64_t wb_layer_bytes, wb_max_outstanding;
  uint32_t n_order;
  const uint32_t* order;
  uint32_t tokens, n_ids, n_pred;
  uint32_t move_bytes;
  uint32_t inclusive; /* dg_inclusive_blocks */
  /* file tier (dg_disk_tier, synchronous reads): blocks = home_blocks + spare blocks; disk[keys] flags the plan's
   * disk units; disk_staging staging buffers (block indices blocks ..); a file read copies the unit's bytes from
   * src_units (keys x unit bytes) when given. xstats (optional): [tokens][6] disk_reads, disk_read_bytes,
   * disk_stage_waits, disk_drops, disk_discards, file-homed units after each boundary. */
  uint32_t disk_tier, disk_prefetch, home_blocks, disk_staging;
  const uint8_t* disk;
  uint64_t* xstats;
  /* reset_at (0 = never): ss_dg_reset_open after the boundary of token reset_at - 1, before that token's table and
   * counters are recorded (the open placement restored, moving only misplaced units); bank_keep: dg_bank_keep (0..2) */
  uint32_t reset_at, bank_keep;
  /* scored eviction: policy 0 LRU, 1 SCORED, 2 SCORED_AUTO; rows = each token's row count at its boundary (0 = 1);
   * weights out of 1000 (all 0 = 700 / 200 / 100); profile (optional): per gated layer units^2 transition counts,
   * row-major [previous unit][unit], loaded as the open state */
  uint32_t policy, rows;
  uint32_t w_trans, w_freq, w_rec, reserved2;
  const uint32_t* profile;
  /* placement rounds: after the boundary of every round_every-th token (0 = never), one round with these limits;
   * rstats (optional): [tokens][6] rounds, promoted to the device, promoted to pinned, demoted from the device,
   * dropped to their file, bytes moved, summed over the rounds so far */
  uint32_t round_every, round_max_units;
  float round_hysteresis, round_decay;
  uint64_t round_budget;
  uint64_t* rstats;
  /* the opt-in policies dg_no_admit, dg_clean_evict, dg_pf_revert_unused, dg_pf_strict_admit (0 / 1); pstats
   * (optional): [tokens][5] clean_drops, clean_drop_bytes, pf_reverted, pf_revert_bytes, pf_strict_refused */
  uint32_t no_admit, clean_evict, pf_revert, pf_strict;
  uint64_t* pstats;
  /* file tier: reads in flight at once (0 / 1 = each inside its fetch); qstats (optional): [tokens][4]
   * disk_overlapped, disk_max_in_flight, disk_carried, disk_carried_bytes */
  uint32_t disk_queue, reserved3;
  uint64_t* qstats;
  /* kept-resident layers: after the boundary of token mr_token[i], event i holds gated layer mr_layer[i]'s units
   * (mr_count[i] ids, the next ones of mr_ids) with ss_dg_make_resident, or releases it (mr_count[i] = 0); a held
   * layer is not exported and its units are kept at every boundary and round. mstats (optional): [tokens][4]
   * resident_units, resident_evicted, mkres_file_reads, mkres_wb_bytes */
  uint32_t mr_n, reserved4;
  const uint32_t* mr_token;
  const uint32_t* mr_layer;
  const uint32_t* mr_count;
  const uint32_t* mr_ids;
  uint64_t* mstats;
  /* sstats (optional): [tokens][5] score_fallbacks, scored_victims, score_layers, score_candidates, score_saturated */
  uint64_t* sstats;
  /* kstats (optional): [tokens][4] bank_kept, bank_keep_drops, bank_keep_rereads, and the FNV-1a 64 hash of the
   * pinned homes' recency order (gated keys as 4 little-endian bytes each, most recently homed first) */
  uint64_t* kstats;
  /* landings: dg_landing_blocks and dg_landing_ttl (the reads are synchronous here); lstats (optional): [tokens][9]
   * landing_issued, landing_promoted, landing_late, landing_expired, landing_dropped_full, landing_read_bytes,
   * landing_expired_layer, landing_skipped_passed, and the units landed or landing after the boundary */
  uint32_t landing_blocks, landing_ttl;
  uint64_t* lstats;
} tsb_dg_replay_config;
SS_API ss_status tsb_test_dg_replay(const tsb_dg_replay_config* cfg, const int32_t* ids, const int32_t* preds,
                                    int32_t* tables, uint64_t* stats, const uint8_t* src_units, uint64_t* read_sum);

/* Test hook: the same configuration and trace driven as the context drives it, with the device's concurrency on the
 * host: three copy streams as worker threads running their copies, entry and ready writes, event records and waits in
 * order after random delays of up to delay_us (seeded), reads in flight landing on their own threads, and an engine
 * thread that exports each layer from the device table as it is, waits for the layer's ready word when its export saw
 * a miss, and reads every routed unit through the device table before it exports the next layer. src_units (required)
 * holds every unit's bytes (unit-major); read_sum[tokens][n_gated][n_ids]: the checksum of each routed unit as the
 * engine read it (0: no entry; the checksum of the deterministic replay). races[5] (may be null): host writes into a
 * block a pending copy reads or writes, host reads of a block a pending copy writes, moves of one wave on a common
 * slot, engine reads of a slot a pending copy writes, copies enqueued on a block whose read has not ended. Decisions
 * that depend on timing may differ from the deterministic replay's; the bytes may not. mutation: 0, or a planted
 * ordering fault of the cache (1: an entry published before its bytes, 2: a demand that does not wait for the prefetch
 * bringing its unit) that the reads and the checks must catch. */
SS_API ss_status tsb_test_dg_async_replay(const tsb_dg_replay_config* cfg, const int32_t* ids, const int32_t* preds,
                                          const uint8_t* src_units, uint32_t seed, uint32_t delay_us, int32_t mutation,
                                          uint64_t* read_sum, uint64_t* races);

/* The device-gated context's slot table as the device holds it (cap >= the gated units; between tokens). Test hook:
 * refused unless the context was opened with dg_test_hooks = 1. */
SS_API ss_status tsb_test_dg_table(ss_ctx* c, int32_t* out, uint32_t cap);

/* Test hook of the landing check: flips the byte at `offset` of the pinned block holding unit (layer, unit) of a
 * device-gated context (the unit must be in pinned RAM, between tokens; refused without dg_test_hooks). A later miss
 * on the unit lands the wrong byte, which the device's check of every landed unit reports at an ss_end (SS_E_HASH) and
 * repairs from the unit's file. */
SS_API ss_status tsb_test_dg_corrupt(ss_ctx* c, int layer, int unit, uint64_t offset);

/* Host forward mode, between ss_acquire and ss_release of `layer` (test hook): per unit of the layer, out[2 u] = where
 * its table entry points (1 = its persistent slot, 2 = a stream ring slot, 0 = no entry) and out[2 u + 1] = that slot
 * (-1 for no entry). n must be the layer's units. */
SS_API ss_status tsb_test_host_locs(ss_ctx* c, int layer, int32_t* out, int n);

/* Host forward mode, between forwards (test and benchmark hook): where unit (layer, unit)'s bytes are kept -
 * *pinned its pinned host block (mapped: kernels can write it at the same address), *device its persistent device
 * slot when it is resident; NULL for either it does not have. A benchmark whose model file is too large for the disk
 * opens on a sparse file and writes every kept unit's bytes here from its generator before the first forward. */
SS_API ss_status tsb_test_host_unit(ss_ctx* c, int layer, int unit, void** pinned, void** device);

/* Test hook: [offset, offset + bytes) of the file at `path` into dst in pieces of `piece` bytes read by a pool of
 * `threads` reader threads (the file tier's reads), unbuffered (O_DIRECT, straight into dst when aligned) when direct
 * is set and the file system allows it. */
SS_API ss_status tsb_test_file_read(const char* path, uint64_t offset, uint64_t bytes, void* dst, uint64_t piece,
                                    uint32_t threads, int direct);

/* Test hook: n reads of `bytes` bytes at offsets[i] of the file at `path` into dst + i x bytes, all begun at once on
 * `threads` reader threads (the file tier's reads in flight), then ended in order (or in reverse); the first failure is
 * returned after every read ended. */
SS_API ss_status tsb_test_async_reads(const char* path, const uint64_t* offsets, uint32_t n, uint64_t bytes, void* dst,
                                      uint32_t threads, int reverse);

/* Test hook: host read-ahead (the host forward mode's readahead_units) on the host alone. Unit u is unit_bytes at
 * offsets[u] of the file at `path` (a read past its end fails with SS_E_IO); `buffers` buffers, `threads` reader
 * threads, each read read_delay_us late. script[n_ops][3] = (op, unit, arg): op 0 requests the unit; op 1 is its
 * fetch: the claim, then, when the claim returns the read, its end and a copy out of the buffer that ends well (arg
 * 0), fails before it started (1) or after (2, the buffer is never reused); op 2 ends the forward; op 3 sleeps arg us.
 * Per fetch: sums[i] = the checksum of the buffer it copied from (0: none), codes[i] = 1 (from the buffer), 0 (the
 * file is read instead) or -status (the read failed after the claim). Per forward end: stats[7] = requested, read,
 * landed, unused, failed, fallbacks so far, bytes read. */
SS_API ss_status tsb_test_read_ahead(const char* path, const uint64_t* offsets, uint32_t n_units, uint64_t unit_bytes,
                                     uint32_t buffers, uint32_t threads, uint32_t read_delay_us, const int32_t* script,
                                     uint32_t n_ops, uint64_t* sums, int32_t* codes, uint64_t* stats);

/* Test hook: the open's fill pipeline on the host alone. Unit i is `unit_bytes` at offsets[i] of the file at `path`;
 * targets[i] >= 0 lands it in slot targets[i] of `device` (a host area standing in for the arena, slots of unit_bytes
 * rounded up to 4 KiB) through a ring of `buffers` buffers of `buffer_bytes`, copied by a copy engine of its own
 * copy_delay_us after each batch was submitted; targets[i] < 0 reads it in place into block -1 - targets[i] of `host`.
 * `readers` reader threads, unbuffered reads when direct is set and allowed. fail_batch >= 0: the copy engine refuses
 * that batch (SS_E_BACKEND). stats[6] (may be null): slot units, in-place units, batches, buffers recycled for a
 * waiting reader, reader waits for a buffer, batches in flight at most. */
SS_API ss_status tsb_test_load(const char* path, const uint64_t* offsets, const int32_t* targets, uint32_t n,
                               uint64_t unit_bytes, void* device, void* host, uint32_t buffers, uint64_t buffer_bytes,
                               uint32_t readers, int direct, uint32_t copy_delay_us, int32_t fail_batch,
                               uint64_t* stats);

/* Test hook: a host-mode resident set (one layer) driven as the host forward mode drives it: n_place units placed at
 * the open (place_pin: pinned), then per step the routed units routed[step][k] (-1 = none) with flags[step][unit]
 * (bit 0: busy, in flight; bit 1: prefetched this forward, so neither a hit nor admitted, a miss for recency), one
 * admission (admit_misses[step], max_ev[step] evictions at most, -1 = no cap) and one observation. Outputs per step:
 * slots_out[step][unit] (-1 = not resident) and counts_out[step][5] (hits, admitted, evicted, transient, deferred).
 * policy: 0 LRU, 1 SCORED with `window` forwards of frequency. */
SS_API ss_status tsb_test_resident_replay(int32_t n_units, int32_t capacity, int32_t policy, uint32_t window,
                                         const int32_t* place_units, const uint8_t* place_pin, uint32_t n_place,
                                         uint32_t steps, const int32_t* routed, uint32_t k, const uint8_t* flags,
                                         const int32_t* max_ev, const uint8_t* admit_misses, int32_t* slots_out,
                                         int32_t* counts_out);

/* Test hook: the device-gated layout ss_open would take for d, p and o (no device work, SS_E_* as ss_open refuses):
 * out[n_out] = keys, R (residents), D (spare slots), B (bank size), P (pinned units), Q (spare blocks), I (inclusive
 * share), F (file units), S (staging buffers), disk_queue, blocks, persistent_slots, slots, guard_slot, unit_bytes,
 * host_stride, disk_tier, disk_prefetch, scored, w_trans, w_freq, w_rec, the resident count (at most 23 values);
 * residents[cap]: the residents' keys. */
SS_API ss_status tsb_test_dg_layout(const ss_desc* d, const ss_plan* p, const ss_options* o, uint64_t* out,
                                    uint32_t n_out, uint32_t* residents, uint32_t cap);

/* Test hooks of scored eviction's profile (the reference's TSSCPRF1 format, ss.h "Scored eviction"): the SHA-256 of
 * len bytes into out[32]; the profile identity of d's gated layers (every layer with units) into identity[32] and,
 * when profile is given, every rule of the format checked (SS_E_INVALID naming the first one broken) and its counts
 * copied into cells (at most cells_cap). */
SS_API ss_status tsb_test_sha256(const void* data, uint64_t len, uint8_t* out);
SS_API ss_status tsb_test_score_profile(const ss_desc* d, const void* profile, uint64_t len, uint8_t* identity,
                                        uint32_t* cells, uint64_t cells_cap);

/* Test hook of the adaptive read depth (dg_disk_queue_adapt): a depth controller of bound `bound` fed n busy periods
 * (reads[i], bytes[i], ns[i]); depth[i] = the depth it returns after period i. params (may be NULL: the defaults
 * 32, 512, 4096, 8192, 0.03, 0.25): min_reads, recheck_u, backoff_1, backoff_max, bar, drift. counters[11] at the end:
 * changes, calibrations, windows, reads at 1, bytes at 1, busy ns at 1, reads at U, bytes at U, busy ns at U,
 * verdicts, calibrating (0 / 1). verdicts[16][7] (may be NULL), the last ones, oldest first: number, reads before it,
 * depth from, depth to, mean rate at U, mean rate at 1 (bytes / ns), reason (0 start, 1 keep U, 2 keep 1, 3 split,
 * 4 recheck, 5 drift); *n_verdicts = how many are filled. */
/* Test hook of the reads-in-flight pool: its scheduling rules checked with a fake read (landing reads behind demand
 * reads, the landing cap and reader reserve, cancel of a landing read not started only, a demand's end running a
 * queued landing read first). SS_OK, or SS_E_BACKEND naming the rule broken. No file, no device. */
SS_API ss_status tsb_test_read_pool(void);
SS_API ss_status tsb_test_read_depth(uint32_t bound, const double* params, uint32_t n, const uint64_t* reads,
                                     const uint64_t* bytes, const uint64_t* ns, uint32_t* depth, uint64_t* counters,
                                     double* verdicts, uint32_t* n_verdicts);

/* ---- Host xxh64 (this library's, the one the open's fill checks pinned units with; seed 0 in the descriptor) ---- */
SS_API uint64_t tsb_xxh64(const void* data, size_t len, uint64_t seed);

/* ---- Build facts ---- */
/* 1000 x major + minor of the CUDA architecture the kernels were compiled for (100 for sm_100a). */
SS_API int tsb_cuda_arch(void);

/* ---- Peer tier (no reference counterpart: the reference declares SS_TIER_PAIR, ss.h:103, and never fetches from
 * it) ----
 * Gated units partitioned over the GPUs' HBM of one box. Each rank's store holds the units it owns (one device
 * allocation, unit i at base + i x unit_bytes, parts back to back); a device-gated miss on an owned unit is copied
 * from its owner's store (over NVLink for a peer, inside HBM for the rank's own) instead of from pinned RAM. The slot
 * cache's decisions are those of pinned RAM (an owned unit keeps its Host home and block number); when every unit is
 * owned, no pinned block is allocated and evictions move no bytes. Keys are gated keys (unit_base[g] + unit). */
#define TSB_PEER_HANDLE_BYTES 64
typedef struct tsb_peer_store tsb_peer_store;

/* owner[keys] from routing counts summed over the ranks (the one exchange step is an all-reduce of these counts):
 * keys in descending count (ties: lower key first), each to the rank with the least count assigned so far (ties:
 * fewer units, then lower rank) among ranks below cap_units[rank] units (NULL: no cap); -1 when every rank is full
 * (the unit stays in pinned RAM). The same counts give the same owners on every rank. */
SS_API ss_status tsb_peer_plan(const uint64_t* counts, uint32_t keys, uint32_t world, const uint64_t* cap_units,
                               int32_t* owner);
/* index[keys]: each owned key's unit index in its owner's store (the owner's keys in key order), -1 if unowned;
 * units_per_rank[world]. Either output may be NULL. */
SS_API ss_status tsb_peer_index(const int32_t* owner, uint32_t keys, uint32_t world, int64_t* index,
                                uint64_t* units_per_rank);
/* This rank's store on `device`: the units with owner[k] == rank read from the descriptor's sources and, with
 * verify and descriptor hashes, checked on the device (K3). An empty store (no unit owned) has a NULL base. */
SS_API ss_status tsb_peer_store_create(const ss_desc* d, const int32_t* owner, uint32_t keys, int32_t rank,
                                       int device, int verify, tsb_peer_store** out);
/* The same store allocated only, for a caller that writes the units itself (its own loader): unit i of the store
 * (tsb_peer_index) at base + i x unit_bytes, its parts back to back in descriptor order; nothing is read or checked. */
SS_API ss_status tsb_peer_store_alloc(const ss_desc* d, const int32_t* owner, uint32_t keys, int32_t rank, int device,
                                      tsb_peer_store** out);
SS_API void tsb_peer_store_free(tsb_peer_store* s);
SS_API void* tsb_peer_store_base(const tsb_peer_store* s);
SS_API uint64_t tsb_peer_store_bytes(const tsb_peer_store* s);
/* The store's CUDA IPC handle (TSB_PEER_HANDLE_BYTES bytes), for the other ranks' processes. */
SS_API ss_status tsb_peer_store_export(const tsb_peer_store* s, void* handle);
/* Maps another process's store on `device` with peer access enabled; *base is its address in this process until
 * tsb_peer_unmap. */
SS_API ss_status tsb_peer_map(const void* handle, int device, void** base);
SS_API ss_status tsb_peer_unmap(void* base);

typedef struct tsb_peer_tier {
  uint32_t struct_size;
  uint32_t world;           /* ranks */
  int32_t rank;             /* this process's rank */
  uint32_t keys;            /* gated keys; owner covers them */
  const int32_t* owner;     /* [keys] owning rank, -1 = pinned RAM */
  void* const* store_base;  /* [world] each rank's store as seen from this process (its own included) */
  uint32_t copy;            /* 0: the land kernel pulls the parts (SM loads), 1: the copy engines */
  uint32_t layout;          /* TSB_PEER_WHOLE_UNITS (0) or TSB_PEER_STRIPED (1): how the stores hold the units */
} tsb_peer_tier;
/* ss_open (device-gated forward mode) with the peer tier. Every store must stay allocated and mapped until
 * ss_close. */
SS_API ss_status tsb_open_peer(const ss_desc* d, const ss_budget* budget, const ss_plan* plan, const ss_options* opt,
                               const tsb_peer_tier* peer, ss_ctx** out);

/* The striped layout (tsb_peer_tier.layout = TSB_PEER_STRIPED): every owned unit is cut into `world` stripes of
 * tsb_peer_stripe_bytes(unit_bytes, world) bytes (ceil(unit_bytes / world) rounded up to 256; the last ones shorter or
 * empty), stripe r covering [r x stripe, min(unit_bytes, (r + 1) x stripe)) of the unit's bytes (parts back to back),
 * and stripe r of every owned unit lives in rank r's store, unit i (its position among all owned keys, key order) at
 * base + i x stripe. A miss then copies 1/world of the unit from every GPU at once (the next rank's stripe first, its
 * own last), so the ranks' pulls are spread over every GPU's links instead of queueing on the owners of the units
 * they miss. The owner map only says which units are in the tier; tsb_peer_store_migrate refuses striped stores (a
 * re-plan that keeps the owned units keeps them as they are). */
#define TSB_PEER_WHOLE_UNITS 0
#define TSB_PEER_STRIPED 1
SS_API uint64_t tsb_peer_stripe_bytes(uint64_t unit_bytes, uint32_t world);
/* This rank's striped store on `device`: stripe `rank` of every unit with owner[k] >= 0, read from the descriptor's
 * sources (fill != 0) or only allocated (fill = 0: the caller writes each stripe at base + i x stripe). NULL base when
 * this rank's stripe is empty or no unit is owned. A stripe is not checked on its own: see tsb_peer_tier_verify. */
SS_API ss_status tsb_peer_store_create_striped(const ss_desc* d, const int32_t* owner, uint32_t keys, int32_t rank,
                                               uint32_t world, int device, int fill, tsb_peer_store** out);
/* The tier against the descriptor's hashes, this rank's share: the owned units whose position among the owned keys is
 * rank modulo world, each gathered whole from the stores as the tier maps them (peers' over NVLink) into scratch on
 * `device` (at most 2 GiB) and hashed there (K3). Call on every rank once every store is written and mapped; together
 * the ranks check each owned unit once, in either layout. SS_E_HASH on a mismatch; checked_units (may be NULL). */
SS_API ss_status tsb_peer_tier_verify(const ss_desc* d, const tsb_peer_tier* peer, int device,
                                      uint64_t* checked_units);

/* Test hook of the striped layout: the copies one owned unit's miss issues on `rank` of `world` (the layout the
 * mover uses: a stripe from every GPU, the next rank's first, each split at the part boundaries it crosses), for a
 * unit of n_parts parts of part_bytes[] bytes; each copy as 5 values: source rank, offset in that rank's stripe,
 * part, offset in the part, bytes. Up to cap copies are written; *n = how many there are. No device. */
SS_API ss_status tsb_test_peer_pieces(const uint64_t* part_bytes, uint32_t n_parts, uint32_t world, int32_t rank,
                                      uint64_t* copies, uint32_t cap, uint32_t* n);

/* A re-plan (after a new all-reduce of routing counts and tsb_peer_plan): dst, allocated by tsb_peer_store_alloc for
 * the new owners, is filled with its units from where they live now (old_owner, old_base[world]: every rank's current
 * store as seen from this process), by the land kernel on `stream` (peers over NVLink, this rank's own store in HBM);
 * returns after the copies landed. A unit unowned before cannot join this way (a new store reads it from its file).
 * Outputs (may be NULL): units copied, of them from peers, bytes. */
SS_API ss_status tsb_peer_store_migrate(tsb_peer_store* dst, const int32_t* old_owner, void* const* old_base,
                                        uint32_t keys, uint32_t world, void* stream, uint64_t* moved_units,
                                        uint64_t* moved_peer_units, uint64_t* moved_bytes);
/* Between tokens: the context's owners and store addresses replaced by `peer` (the same world, rank and set of owned
 * units; only owners change). Every copy that read the old stores has finished when it returns, so every rank may
 * release its old stores once all ranks returned from this call. */
SS_API ss_status tsb_dg_peer_retier(ss_ctx* c, const tsb_peer_tier* peer);

#ifdef __cplusplus
}
#endif

#endif /* TIERSTREAM_TSB_H */
