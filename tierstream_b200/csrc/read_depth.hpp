// dg_disk_queue_adapt: how many demand file reads the read pool runs at once, 1 or its bound U (the readers stay
// allocated at U), chosen from measured throughput (the reference's DgDepthCtl, src/dg_load.hpp:151-206 and
// src/dg_load.cpp:579-674; its rules restated here).
//
// The pool reports one busy period at a time (from idle to idle: in demand-only decoding, one layer's file reads):
// the reads that ended in it, their bytes and its wall time. Periods add up into windows of at least min_reads
// reads, and a window's rate is its bytes / ns. A calibration measures four windows at U, 1, 1, U: U is kept only if
// both brackets (window 0 against 1, window 3 against 2) show it at least `bar` faster; a split verdict is measured
// once more, then settles on 1. Held at U, the depth is calibrated again after recheck_u reads; held at 1, after
// backoff_1 reads the first time and backoff_max reads while U keeps losing. While held, two windows in a row more
// than `drift` away from the held depth's calibrated rate start a calibration at once. No clock and no thread: the
// pool measures, so the decisions are a function of the periods it is fed.
#pragma once

#include <cstdint>
#include <vector>

namespace tsb {

class ReadDepth {
 public:
  struct Params {
    uint64_t min_reads = 32, recheck_u = 512, backoff_1 = 4096, backoff_max = 8192;
    double bar = 0.03, drift = 0.25;
  };
  enum Why : uint8_t { kStart = 0, kKeepU, kKeep1, kSplit, kRecheck, kDrift };
  struct Verdict {  // one calibration's outcome, kept in a ring of the last kKept
    uint64_t seq = 0, reads = 0;    // its number; the reads ended before it
    uint32_t from = 0, to = 0;      // the depth before and after
    double rate_u = 0, rate_1 = 0;  // the calibration's mean window rates at U and at 1 (bytes / ns)
    Why why = kStart;
  };
  static constexpr size_t kKept = 16;

  ReadDepth(uint32_t bound, const Params& p);
  explicit ReadDepth(uint32_t bound) : ReadDepth(bound, Params{}) {}
  // A busy period at depth() ended after `reads` reads of `bytes` bytes in `ns`: the depth for the next one.
  uint32_t on_busy(uint64_t reads, uint64_t bytes, uint64_t ns);
  uint32_t depth() const { return depth_; }
  uint32_t bound() const { return bound_; }
  bool calibrating() const { return window_at_ < 4; }
  uint64_t verdicts() const { return verdicts_; }
  const std::vector<Verdict>& recent() const { return recent_; }  // oldest first

  // depth changes, calibrations begun, windows closed; reads, bytes and busy ns at depth 1 and at U
  uint64_t changes = 0, calibrations = 0, windows = 0;
  uint64_t reads_1 = 0, bytes_1 = 0, ns_1 = 0, reads_u = 0, bytes_u = 0, ns_u = 0;

 private:
  void start_calibration(Why why);
  void go(uint32_t d);
  void settle();
  void remember(const Verdict& v);

  Params p_;
  uint32_t bound_, depth_;
  uint32_t window_at_ = 0;  // 0..3: the calibration window being measured; 4: holding
  bool again_ = false;      // the running calibration repeats a split one
  double rate_[4] = {0, 0, 0, 0};
  double held_rate_ = 0;
  uint32_t far_in_a_row_ = 0;
  uint64_t w_reads_ = 0, w_bytes_ = 0, w_ns_ = 0;  // the open window
  uint64_t reads_ = 0, held_reads_ = 0, hold_for_ = 0, next_backoff_ = 0;
  uint64_t verdicts_ = 0;
  std::vector<Verdict> recent_;
};

}  // namespace tsb
