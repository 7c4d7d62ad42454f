/* C interface of the reference harness (oracle/_ref/libtsref.so, built by oracle/Makefile from the reference's own
 * sources). TEST INFRASTRUCTURE ONLY: the tests, smoke() and bench.py's cpu_baseline leg use it as the checker; the
 * product library never links or calls it. */
#ifndef TSB_OREF_H
#define TSB_OREF_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct oref_dg_config {
  uint32_t n_gated;
  const uint32_t* n_units;      /* [n_gated] */
  uint32_t n_parts;
  const uint64_t* part_bytes;   /* [n_parts] */
  uint32_t persistent_slots, bank_slots, blocks, spare_target;
  uint32_t prefetch_reserve;    /* 0xFFFFFFFF = auto, min(24, spare_target / 4) */
  uint32_t prefetch_per_layer, prefetch_per_token;
  uint32_t wb_defer, wb_on_d2h;
  uint64_t wb_layer_bytes, wb_max_outstanding;
  uint32_t n_order;
  const uint32_t* order;        /* placement priority (keys) */
  uint32_t tokens, n_ids, n_pred; /* ids: [tokens][n_gated][n_ids]; preds: [tokens][n_gated][n_pred] (for g + 1) */
  uint32_t move_bytes;          /* 1 = the transport moves real bytes (host arena and blocks); 2 = timing sample:
                                   real copies into 4 aliased unit buffers each for slots and blocks */
  uint32_t inclusive;           /* dg_inclusive_blocks (the clean-copy share) */
  /* three-tier (dg_disk_tier, synchronous reads: disk_queue 1): blocks = home_blocks + spare blocks; disk[keys] = 1 for
   * the plan's disk units; disk_staging staging buffers; a read copies src_units' bytes when given. xstats (optional):
   * [tokens][OREF_NXSTATS] disk_reads, disk_read_bytes, disk_stage_waits, disk_drops, disk_discards, file units. */
  uint32_t disk_tier, disk_prefetch, home_blocks, disk_staging;
  const uint8_t* disk;
  uint64_t* xstats;
  uint32_t reset_at, bank_keep; /* reset_at (0 = never): reset_open after the boundary of token reset_at - 1;
                                   bank_keep: dg_bank_keep (0..2) */
  /* scored eviction: policy 0 LRU / 1 SCORED / 2 SCORED_AUTO, rows per boundary (0 = 1), weights out of 1000 (all 0 =
   * the defaults), profile (optional): per gated layer units^2 counts, loaded through a TSSCPRF1 profile */
  uint32_t policy, rows;
  uint32_t w_trans, w_freq, w_rec, reserved2;
  const uint32_t* profile;
  /* placement rounds after the boundary of every round_every-th token (0 = never); rstats (optional): [tokens][6]
   * rounds, promoted to device, promoted to pinned, demoted, dropped to file, bytes, summed so far */
  uint32_t round_every, round_max_units;
  float round_hysteresis, round_decay;
  uint64_t round_budget;
  uint64_t* rstats;
  /* opt-in policies (0 / 1); pstats (optional): [tokens][5] clean_drops, clean_drop_bytes, pf_reverted,
   * pf_revert_bytes, pf_strict_refused */
  uint32_t no_admit, clean_evict, pf_revert, pf_strict;
  uint64_t* pstats;
  /* three-tier reads in flight (0 / 1 = synchronous); qstats (optional): [tokens][4] disk_overlapped,
   * disk_max_in_flight, disk_carried, disk_carried_bytes */
  uint32_t disk_queue, reserved3;
  uint64_t* qstats;
  /* kept-resident layers: make_resident events after the boundary of mr_token[i] (mr_count[i] = 0: a release);
   * mstats (optional): [tokens][4] resident_units, resident_evicted, mkres_file_reads, mkres_wb_bytes */
  uint32_t mr_n, reserved4;
  const uint32_t* mr_token;
  const uint32_t* mr_layer;
  const uint32_t* mr_count;
  const uint32_t* mr_ids;
  uint64_t* mstats;
  /* sstats (optional): [tokens][5] score_fallbacks, scored_victims, score_layers, score_candidates, score_saturated */
  uint64_t* sstats;
  /* kstats (optional): [tokens][4] bank_kept, bank_keep_drops, bank_keep_rereads, FNV-1a 64 of the pinned homes'
   * recency order (keys as 4 little-endian bytes, most recently homed first) */
  uint64_t* kstats;
  /* landings (dg_landing_blocks, dg_landing_ttl; synchronous reads); lstats (optional): [tokens][9] landing_issued,
   * landing_promoted, landing_late, landing_expired, landing_dropped_full, landing_read_bytes, landing_expired_layer,
   * landing_skipped_passed, units landed or landing */
  uint32_t landing_blocks, landing_ttl;
  uint64_t* lstats;
} oref_dg_config;
#define OREF_NXSTATS 6

/* Counters dumped per token (in this order). */
#define OREF_NSTATS 16
/* tokens, lookups, misses, covered, fetched, prefetched, prefetch_used, resurrected, bank_serves, collected_mid,
 * evicted, evict_short, writebacks_done, wb_deferred, wb_cancelled, wb_forced */

/* Replays the trace through the reference DgCore in the service thread's order with a host transport whose events are
 * always complete. tables: [tokens][keys] slot_of after each boundary; stats: [tokens][OREF_NSTATS]. When move_bytes
 * and src_units (keys x unit_bytes, each unit's bytes) are given, read_sum receives per (token, g, id) the checksum
 * sum(byte * (pos % 251 + 1)) of the bytes found through the slot table after the layer's demand (0 for an absent
 * entry). Returns 0, or -1 with the message in err. */
/* The reference's adaptive read depth controller fed n busy periods (reads, bytes, ns); the outputs of the library's
 * tsb_test_read_depth. params (may be NULL): min_reads, recheck_u, backoff_1, backoff_max, bar, drift. */
int oref_read_depth(uint32_t bound, const double* params, uint32_t n, const uint64_t* reads, const uint64_t* bytes,
                    const uint64_t* ns, uint32_t* depth, uint64_t* counters, double* verdicts, uint32_t* n_verdicts);
int oref_dg_replay(const oref_dg_config* cfg, const int32_t* ids, const int32_t* preds, int32_t* tables,
                   uint64_t* stats, const uint8_t* src_units, uint64_t* read_sum, char* err, size_t errlen);

/* Reference xxh64 (the reference's own xxh64.cpp). */
uint64_t oref_xxh64(const void* data, size_t len, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
