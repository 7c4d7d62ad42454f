// Host read-ahead for the host forward mode (readahead_units > 0; the reference's, src/stream_ctx.cpp:726-1021,
// 1401-1448, 1600-1632): file-backed units the engine expects (ss_host_prefetch, ss_host_prefetch_layer, and units
// left waiting for a ring slot) are read from their files into a set of pinned host buffers ahead of their fetch, so
// the fetch copies from host memory instead of reading the file then.
//
// Per forward each unit is requested at most once; a request starts reading as soon as a buffer is free (oldest
// request first) on this object's reader threads. A unit's fetch claims its entry: a request not started yet is
// abandoned and the fetch reads the file as usual; a read that failed before the claim is a fallback to the file; a
// read running or finished is the fetch's source: the fetch waits for the read's end and copies out of the buffer
// (a read that fails after the claim fails the fetch with the read's error, as a file read would). The buffer comes
// back when the fetch's copy ended, or at the forward's end for a read nobody claimed; a buffer whose copy failed
// after it started is never reused. At the forward's end every read has ended, unclaimed requests are dropped, and
// each entry is counted once: requested, read (finished), landed (copied to the device), unused (read, never copied),
// failed (read failed), with the bytes read; fallbacks are counted at the claim.
#pragma once

#include <condition_variable>
#include <cstdint>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "strix_stream/ss.h"

namespace tsb {

struct RaStats {
  uint64_t requested = 0, read = 0, landed = 0, unused = 0, failed = 0, fallback = 0, bytes = 0;
};

class ReadAhead {
 public:
  struct Entry {
    enum St { Waiting, Reading, Ready, Landing, Consumed, Failed, Abandoned };
    St st = Waiting;
    int layer = 0, unit = 0;
    int32_t buf = -1;               // the buffer it holds (-1: none)
    bool started = false, ended = false, ok = false, quarantined = false;
    uint64_t bytes = 0;             // read from the file
    ss_status err = SS_OK;
    std::string msg;
  };
  using EntryPtr = std::shared_ptr<Entry>;
  // read(layer, unit, dst): the unit's bytes from its file into dst, checked; returns the bytes read; throws on failure.
  using Read = std::function<uint64_t(int, int, char*)>;

  ReadAhead(std::vector<char*> buffers, unsigned threads, Read read);
  ~ReadAhead();
  ReadAhead(const ReadAhead&) = delete;
  ReadAhead& operator=(const ReadAhead&) = delete;

  bool requested(int layer, int unit) const;
  void request(int layer, int unit);     // ignored when already requested this forward or during end_forward
  EntryPtr claim(int layer, int unit);   // the unit's fetch; nullptr: read its file
  // The claimed read's end: its buffer, or nullptr with the read's error in *status / *msg.
  const char* wait(Entry& e, ss_status* status, std::string* msg);
  // The fetch's copy out of the buffer ended (ok), or failed before (issued = false) or after it started copying.
  void done(Entry& e, bool ok, bool issued);
  RaStats end_forward();                 // after every fetch of the forward ended
  RaStats totals() const;
  size_t buffers() const { return bufs_.size(); }

 private:
  static uint64_t key(int layer, int unit) { return (uint64_t(uint32_t(layer)) << 32) | uint32_t(unit); }
  void start_locked();                   // waiting requests onto free buffers
  void give_back_locked(Entry& e);
  void loop();

  std::vector<char*> bufs_;
  Read read_;
  mutable std::mutex mu_;
  std::condition_variable cv_;
  std::unordered_map<uint64_t, EntryPtr> entries_;  // this forward's
  std::deque<EntryPtr> waiting_, queue_;            // not yet given a buffer; given one, not yet taken by a reader
  std::vector<int32_t> free_;
  unsigned running_ = 0;
  bool frozen_ = false, stop_ = false;
  RaStats total_;
  std::vector<std::thread> th_;
};

}  // namespace tsb
