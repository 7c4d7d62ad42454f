"""The device-gated decode's cost per layer when nothing misses (north star: under 5 us per layer).

A small gated model with every unit resident; two graphs captured on one stream: (A) the token step an engine runs
(begin, per layer export -> wait -> reader of the routed units, end) and (B) the same reader kernels alone. Per token,
the device time of A (inside ss_begin / ss_end) minus the device time of B, divided by the layers, is what the
device-gated protocol adds to a layer. Also reported: A with no reader at all (the protocol's kernels back to back).

    python -m tierstream_b200.dg_overhead [--layers 32] [--tokens 200]
"""
import argparse
import ctypes as C
import json
import os

import numpy as np
import torch

from . import abi, harness, runtime, synth


def measure(layers=32, units=8, part=256 << 10, top_k=2, tokens=200, warmup=20):
    m = synth.Model(os.path.join(harness.model_dir(), "tsb-overhead-%d.bin" % layers), layers=layers, units=units,
                    part_bytes=(part, part, part), seed=9, top_k=top_k)
    m.write()
    run = harness.DgRun(m, residents_per_layer=units - 1, spare_per_layer=1, max_ids=top_k, test_hooks=False,
                        mode=1, slices=8)
    eng = abi.load_engine()
    try:
        # routes only to residents (units 0 .. units - 2 of every layer): no token ever misses, so no wait kernel
        # ever waits on the service (the run also works under a profiler that serialises kernels)
        ids = np.tile(np.arange(top_k, dtype=np.int32), (layers, 1))
        run.ids_pin.numpy()[:] = ids.reshape(-1)
        run.ids_dev.copy_(run.ids_pin)
        for _ in range(3):
            run.step(ids)
        s = run.stream
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

        def time_a(graph):
            tot = 0.0
            for t in range(warmup + tokens):
                run.ctx.begin()
                e0.record(s)
                graph.launch()
                e1.record(s)
                run.ctx.end()
                e1.synchronize()
                if t >= warmup:
                    tot += e0.elapsed_time(e1)
            return tot * 1000 / tokens  # us per token

        st0 = run.ctx.stats()
        a_us = time_a(run.graph)
        st1 = run.ctx.stats()
        assert st1["misses"] == st0["misses"], "the overhead run must not miss"
        bare = runtime.TokenGraph(run.ctx, layers, run.ids_dev.data_ptr(), top_k, run.out_dev.data_ptr(),
                                  s.cuda_stream, slices=8, mode=1, with_reader=False)
        bare_us = time_a(bare)
        bare.close()
        # (B) the readers alone, captured into a graph of their own
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
            for L in range(layers):
                eng.tse_read_units(run.ctx.h, L, run.ids_dev.data_ptr() + 4 * L * top_k, top_k,
                                   run.out_dev.data_ptr() + 8 * L * top_k, 8, 1, s.cuda_stream)
        tot = 0.0
        for t in range(warmup + tokens):
            e0.record(s)
            g.replay()
            e1.record(s)
            e1.synchronize()
            if t >= warmup:
                tot += e0.elapsed_time(e1)
        b_us = tot * 1000 / tokens
        return {"layers": layers, "token_us_with_protocol": round(a_us, 2), "token_us_readers_only": round(b_us, 2),
                "overhead_us_per_layer": round((a_us - b_us) / layers, 3),
                "protocol_only_us_per_layer": round(bare_us / layers, 3)}
    finally:
        run.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--tokens", type=int, default=200)
    a = ap.parse_args()
    print(json.dumps(measure(layers=a.layers, tokens=a.tokens)))


if __name__ == "__main__":
    main()
