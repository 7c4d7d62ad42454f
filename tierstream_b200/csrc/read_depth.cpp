#include "read_depth.hpp"

#include <algorithm>

namespace tsb {

ReadDepth::ReadDepth(uint32_t bound, const Params& p) : p_(p), bound_(std::max<uint32_t>(bound, 1)), depth_(bound_) {
  if (p_.min_reads == 0) p_.min_reads = 1;
  next_backoff_ = p_.backoff_1;
  start_calibration(kStart);
}

void ReadDepth::go(uint32_t d) {
  changes += d != depth_ ? 1 : 0;
  depth_ = d;
}

// Four windows from here: at U, 1, 1, U.
void ReadDepth::start_calibration(Why) {
  window_at_ = 0;
  ++calibrations;
  go(bound_);
  w_reads_ = w_bytes_ = w_ns_ = 0;
}

void ReadDepth::remember(const Verdict& v) {
  if (recent_.size() == kKept) recent_.erase(recent_.begin());
  recent_.push_back(v);
}

// The four windows measured: keep U, settle on 1, or (a first split verdict) measure once more.
void ReadDepth::settle() {
  const double lift = 1.0 + p_.bar;
  const bool first_says_u = rate_[0] >= lift * rate_[1];
  const bool second_says_u = rate_[3] >= lift * rate_[2];
  Verdict v;
  v.seq = ++verdicts_;
  v.reads = reads_;
  v.from = depth_;
  v.rate_u = (rate_[0] + rate_[3]) / 2;
  v.rate_1 = (rate_[1] + rate_[2]) / 2;
  if (first_says_u != second_says_u && !again_) {
    again_ = true;
    v.to = bound_;
    v.why = kSplit;
    remember(v);
    start_calibration(kSplit);
    --calibrations;  // (a repeat of the same calibration, not a new one)
    return;
  }
  again_ = false;
  const bool keep_u = first_says_u && second_says_u;
  v.to = keep_u ? bound_ : 1u;
  v.why = keep_u ? kKeepU : kKeep1;
  remember(v);
  window_at_ = 4;
  far_in_a_row_ = 0;
  held_reads_ = 0;
  held_rate_ = keep_u ? v.rate_u : v.rate_1;
  if (keep_u) {
    hold_for_ = p_.recheck_u;
    next_backoff_ = p_.backoff_1;  // U won: a later loss backs off from the start again
  } else {
    hold_for_ = next_backoff_;
    next_backoff_ = p_.backoff_max;
  }
  go(keep_u ? bound_ : 1u);
}

uint32_t ReadDepth::on_busy(uint64_t reads, uint64_t bytes, uint64_t ns) {
  if (bound_ <= 1 || reads == 0) return depth_;
  reads_ += reads;
  if (depth_ == 1) {
    reads_1 += reads;
    bytes_1 += bytes;
    ns_1 += ns;
  } else {
    reads_u += reads;
    bytes_u += bytes;
    ns_u += ns;
  }
  w_reads_ += reads;
  w_bytes_ += bytes;
  w_ns_ += ns;
  if (window_at_ == 4) held_reads_ += reads;
  if (w_reads_ < p_.min_reads) return depth_;
  const double rate = w_ns_ ? double(w_bytes_) / double(w_ns_) : 0.0;
  w_reads_ = w_bytes_ = w_ns_ = 0;
  ++windows;
  if (window_at_ < 4) {  // calibrating: this window's rate, then the next window's depth (U, 1, 1, U)
    rate_[window_at_++] = rate;
    if (window_at_ == 4) settle();
    else go(window_at_ == 3 ? bound_ : 1u);
    return depth_;
  }
  // holding: a drift (two far windows in a row) or a due re-check starts a calibration
  const bool far = held_rate_ > 0 && (rate > held_rate_ * (1 + p_.drift) || rate < held_rate_ * (1 - p_.drift));
  far_in_a_row_ = far ? far_in_a_row_ + 1 : 0;
  if (far_in_a_row_ >= 2) start_calibration(kDrift);
  else if (held_reads_ >= hold_for_) start_calibration(kRecheck);
  return depth_;
}

}  // namespace tsb
