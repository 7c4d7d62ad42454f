// Times the reference library's own CUDA device-gated decode (BENCHMARK INFRASTRUCTURE, for context only: bench.py
// --impl reference-cuda runs it; the product never links it). Built by oracle/Makefile from the reference's sources
// with its CUDA backend (REF/src with SS_WITH_CUDA, REF/src/dg_kernels.cu for sm_100a: the reference's export, wait
// and end kernels, its ready word in mapped host memory) and this repository's engine stand-in
// (tierstream_b200/csrc/engine_sim.cu, which uses only the ss.h ABI), so the token graph is the one bench.py captures
// on this library, captured on the reference's context.
//
//   ref_dg_cuda stream DIR WARMUP STEPS SLICES   one JSON line: the expert-miss stream of STEPS timed tokens and the
//                                                readers' checksums compared with DIR/want.u64
//   ref_dg_cuda zero DIR TOKENS                  one JSON line: the protocol's cost per layer when nothing misses
//
// DIR holds desc.json, tiers.u8, budget.bin and options.bin (ss_budget / ss_options as bytes), meta.txt ("G U N"
// gated layers, units per layer, ids per layer), ids.i32 ([tokens][G][N]) and, for stream, want.u64 (word-sum
// checksum per key).
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "strix_stream/ss.h"

extern "C" {
int tse_capture_token(ss_ctx* c, uint32_t n_gated, const int32_t* ids_dev, uint32_t n_ids, const int32_t* pred_dev,
                      uint32_t n_pred, unsigned long long* out_dev, uint32_t slices, int mode, int with_reader,
                      void* stream, void** exec_out, const uint8_t* held);
int tse_launch(void* exec, void* stream);
int tse_destroy(void* exec);
int tse_read_units(ss_ctx* c, uint32_t g, const int32_t* ids_dev, uint32_t n, unsigned long long* out_dev,
                   uint32_t slices, int mode, void* stream);
}

namespace {

[[noreturn]] void die(const std::string& what) {
  std::printf("{\"error\": \"%s\"}\n", what.c_str());
  std::exit(2);
}
void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) die(std::string(what) + ": " + cudaGetErrorString(e));
}
void ok(ss_status s, const char* what) {
  if (s != SS_OK) die(std::string(what) + ": " + ss_last_error());
}
void rc(int r, const char* what) {
  if (r != 0) die(std::string(what) + " returned " + std::to_string(r) + (r >= 1000 ? std::string(": ") + ss_last_error() : ""));
}
std::string slurp(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) die("cannot read " + path);
  std::ostringstream s;
  s << f.rdbuf();
  return s.str();
}

struct Opened {
  ss_desc* d = nullptr;
  ss_plan* p = nullptr;
  ss_ctx* c = nullptr;
  uint32_t G = 0, U = 0, N = 0;
  uint64_t unit_bytes = 0;
  std::vector<int32_t> ids;
};

Opened open_dir(const std::string& dir) {
  Opened o;
  std::istringstream meta(slurp(dir + "/meta.txt"));
  meta >> o.G >> o.U >> o.N;
  const std::string desc = slurp(dir + "/desc.json"), tiers = slurp(dir + "/tiers.u8");
  const std::string bud = slurp(dir + "/budget.bin"), opt = slurp(dir + "/options.bin");
  if (bud.size() != sizeof(ss_budget) || opt.size() != sizeof(ss_options)) die("budget / options size");
  ss_budget b;
  ss_options op;
  std::memcpy(&b, bud.data(), sizeof b);
  std::memcpy(&op, opt.data(), sizeof op);
  ok(ss_desc_from_json(desc.data(), desc.size(), &o.d), "ss_desc_from_json");
  ok(ss_plan_from_tiers(o.d, &b, reinterpret_cast<const uint8_t*>(tiers.data()), tiers.size(), &o.p),
     "ss_plan_from_tiers");
  ok(ss_open(o.d, &b, o.p, &op, &o.c), "ss_open");
  o.unit_bytes = ss_desc_unit_bytes(o.d, 0);
  const std::string ids = slurp(dir + "/ids.i32");
  o.ids.resize(ids.size() / 4);
  std::memcpy(o.ids.data(), ids.data(), ids.size());
  return o;
}

uint64_t landed(ss_ctx* c) {
  ss_dg_stats s;
  ok(ss_stats_dg_sized(c, &s, sizeof s), "ss_stats_dg");
  return s.fetched + s.prefetched;
}

int stream_mode(const std::string& dir, int warmup, int steps, uint32_t slices) {
  Opened o = open_dir(dir);
  const size_t cells = size_t(o.G) * o.N;
  if (o.ids.size() < size_t(warmup + steps) * cells) die("ids.i32 holds fewer tokens than warmup + steps");
  const std::string want_raw = slurp(dir + "/want.u64");
  std::vector<uint64_t> want(want_raw.size() / 8);
  std::memcpy(want.data(), want_raw.data(), want_raw.size());
  cudaStream_t s;
  ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
  int32_t *trace = nullptr, *ids = nullptr;
  unsigned long long *out = nullptr, *outs = nullptr;
  ck(cudaMalloc(&trace, o.ids.size() * 4), "malloc");
  ck(cudaMalloc(&ids, cells * 4), "malloc");
  ck(cudaMalloc(&out, cells * 8), "malloc");
  ck(cudaMalloc(&outs, size_t(steps) * cells * 8), "malloc");
  ck(cudaMemcpy(trace, o.ids.data(), o.ids.size() * 4, cudaMemcpyHostToDevice), "trace upload");
  void* exec = nullptr;
  rc(tse_capture_token(o.c, o.G, ids, o.N, nullptr, 0, out, slices, 1, 1, s, &exec, nullptr), "tse_capture_token");
  auto token = [&](int t) {
    ok(ss_begin(o.c, nullptr, 0), "ss_begin");
    ck(cudaMemcpyAsync(ids, trace + size_t(t) * cells, cells * 4, cudaMemcpyDeviceToDevice, s), "ids");
    rc(tse_launch(exec, s), "graph launch");
  };
  for (int t = 0; t < warmup; ++t) {
    token(t);
    ok(ss_end(o.c), "ss_end");
  }
  ck(cudaStreamSynchronize(s), "sync");
  const uint64_t u0 = landed(o.c);
  cudaEvent_t e0, e1;
  ck(cudaEventCreate(&e0), "event");
  ck(cudaEventCreate(&e1), "event");
  ck(cudaEventRecord(e0, s), "record");
  for (int t = 0; t < steps; ++t) {
    token(warmup + t);
    ck(cudaMemcpyAsync(outs + size_t(t) * cells, out, cells * 8, cudaMemcpyDeviceToDevice, s), "outs");
    ok(ss_end(o.c), "ss_end");
  }
  ck(cudaEventRecord(e1, s), "record");
  ck(cudaEventSynchronize(e1), "sync");
  float ms = 0;
  ck(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
  const uint64_t units = landed(o.c) - u0;
  std::vector<unsigned long long> got(size_t(steps) * cells);
  ck(cudaMemcpy(got.data(), outs, got.size() * 8, cudaMemcpyDeviceToHost), "outs download");
  uint64_t bad = 0;
  for (int t = 0; t < steps; ++t)
    for (uint32_t g = 0; g < o.G; ++g)
      for (uint32_t i = 0; i < o.N; ++i) {
        const size_t k = size_t(warmup + t) * cells + size_t(g) * o.N + i;
        const uint64_t key = uint64_t(g) * o.U + uint64_t(o.ids[k]);
        bad += got[size_t(t) * cells + size_t(g) * o.N + i] != want[key] ? 1 : 0;
      }
  ss_dg_stats st;
  ok(ss_stats_dg_sized(o.c, &st, sizeof st), "ss_stats_dg");
  std::printf("{\"value\": %.3f, \"ms_per_step\": %.3f, \"units_landed\": %llu, \"unit_bytes\": %llu, "
              "\"tokens\": %d, \"reads\": %zu, \"mismatches\": %llu, \"misses\": %llu, \"lookups\": %llu}\n",
              double(units) * double(o.unit_bytes) / (double(ms) / 1e3) / 1e9, double(ms) / steps,
              (unsigned long long)units, (unsigned long long)o.unit_bytes, steps, got.size(),
              (unsigned long long)bad, (unsigned long long)st.misses, (unsigned long long)st.lookups);
  tse_destroy(exec);
  ss_close(o.c);
  ss_plan_free(o.p);
  ss_desc_free(o.d);
  return bad ? 1 : 0;
}

// As tierstream_b200/dg_overhead.py: (A) the token graph inside ss_begin / ss_end, (bare) the same without readers,
// (B) the readers alone in a graph of their own; per layer (A - B) / G.
int zero_mode(const std::string& dir, int tokens) {
  Opened o = open_dir(dir);
  const size_t cells = size_t(o.G) * o.N;
  cudaStream_t s;
  ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
  int32_t* ids = nullptr;
  unsigned long long* out = nullptr;
  ck(cudaMalloc(&ids, cells * 4), "malloc");
  ck(cudaMalloc(&out, cells * 8), "malloc");
  ck(cudaMemcpy(ids, o.ids.data(), cells * 4, cudaMemcpyHostToDevice), "ids");
  void *a = nullptr, *bare = nullptr;
  rc(tse_capture_token(o.c, o.G, ids, o.N, nullptr, 0, out, 8, 1, 1, s, &a, nullptr), "capture");
  rc(tse_capture_token(o.c, o.G, ids, o.N, nullptr, 0, out, 8, 1, 0, s, &bare, nullptr), "capture");
  cudaEvent_t e0, e1;
  ck(cudaEventCreate(&e0), "event");
  ck(cudaEventCreate(&e1), "event");
  const int warm = 20;
  ss_dg_stats s0;
  ok(ss_stats_dg_sized(o.c, &s0, sizeof s0), "stats");
  auto time_tokens = [&](void* g) {
    double tot = 0;
    for (int t = 0; t < warm + tokens; ++t) {
      ok(ss_begin(o.c, nullptr, 0), "ss_begin");
      ck(cudaEventRecord(e0, s), "record");
      rc(tse_launch(g, s), "launch");
      ck(cudaEventRecord(e1, s), "record");
      ok(ss_end(o.c), "ss_end");
      ck(cudaEventSynchronize(e1), "sync");
      float ms = 0;
      ck(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
      if (t >= warm) tot += ms;
    }
    return tot * 1000 / tokens;
  };
  const double a_us = time_tokens(a), bare_us = time_tokens(bare);
  ss_dg_stats s1;
  ok(ss_stats_dg_sized(o.c, &s1, sizeof s1), "stats");
  if (s1.misses != s0.misses) die("the zero-miss run missed");
  cudaGraph_t graph = nullptr;
  ck(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "capture");
  for (uint32_t g = 0; g < o.G; ++g) rc(tse_read_units(o.c, g, ids + size_t(g) * o.N, o.N, out + size_t(g) * o.N, 8, 1, s), "reader");
  ck(cudaStreamEndCapture(s, &graph), "capture");
  cudaGraphExec_t rd = nullptr;
  ck(cudaGraphInstantiate(&rd, graph, 0), "instantiate");
  double tot = 0;
  for (int t = 0; t < warm + tokens; ++t) {
    ck(cudaEventRecord(e0, s), "record");
    ck(cudaGraphLaunch(rd, s), "launch");
    ck(cudaEventRecord(e1, s), "record");
    ck(cudaEventSynchronize(e1), "sync");
    float ms = 0;
    ck(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
    if (t >= warm) tot += ms;
  }
  const double b_us = tot * 1000 / tokens;
  std::printf("{\"layers\": %u, \"token_us_with_protocol\": %.2f, \"token_us_readers_only\": %.2f, "
              "\"overhead_us_per_layer\": %.3f, \"protocol_only_us_per_layer\": %.3f}\n",
              o.G, a_us, b_us, (a_us - b_us) / o.G, bare_us / o.G);
  cudaGraphExecDestroy(rd);
  cudaGraphDestroy(graph);
  tse_destroy(a);
  tse_destroy(bare);
  ss_close(o.c);
  ss_plan_free(o.p);
  ss_desc_free(o.d);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc >= 6 && !std::strcmp(argv[1], "stream"))
    return stream_mode(argv[2], std::atoi(argv[3]), std::atoi(argv[4]), uint32_t(std::atoi(argv[5])));
  if (argc >= 4 && !std::strcmp(argv[1], "zero")) return zero_mode(argv[2], std::atoi(argv[3]));
  std::fprintf(stderr, "usage: ref_dg_cuda stream DIR WARMUP STEPS SLICES | zero DIR TOKENS\n");
  return 2;
}
