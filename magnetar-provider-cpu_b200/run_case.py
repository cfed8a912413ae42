#!/usr/bin/env python
"""Times one packed matmul shape on one GPU, for profiling and sweeps.

    python magnetar-provider-cpu_b200/run_case.py --fmt q4_k --m 1 --n 28672 --k 8192 \
        [--launches 200] [--copies 0] [--graph] [--min-workspace]

Each launch is one `mgb_qmatmul` (x [m, k] f32 -> y [m, n] f32) on its own
weight copy, rotating over enough device copies to exceed 3x the 126 MB L2
(`--copies` overrides).  With `--graph` the launches are captured once as a
CUDA graph of back-to-back calls and the graph is replayed (the way a decode
step issues them); otherwise they are launched from the host.  Prints one
JSON line: device time per launch (CUDA events on the launching stream), the
weight bytes per launch and the algorithmic GB/s (packed weights + x + y) and
TFLOP/s.  Under ncu, pass `--launches` small and `-s/-c` to ncu.
"""

from __future__ import annotations

import argparse
import json
import pathlib
import sys
import time

HERE = pathlib.Path(__file__).resolve().parent
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))

import magnetar_b200 as mgb  # noqa: E402
import synthetic  # noqa: E402

FORMATS = {"q4_k": mgb.Q4_K, "q5_k": mgb.Q5_K, "q6_k": mgb.Q6_K, "q8_0": mgb.Q8_0,
           "iq4_nl": mgb.IQ4_NL, "q4_0": mgb.Q4_0}
L2_BYTES = 126 * 1024 * 1024


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--fmt", default="q4_k", choices=sorted(FORMATS))
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--launches", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--copies", type=int, default=0)
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--min-workspace", action="store_true")
    args = ap.parse_args()

    import torch

    fmt, m, n, k = FORMATS[args.fmt], args.m, args.n, args.k
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream()
    wb = mgb.packed_bytes(fmt, n, k)
    copies = args.copies or max(2, -(-3 * L2_BYTES // (wb + 4 * m * (n + k))))
    src = torch.from_numpy(synthetic.packed_weights(fmt, n, k)).to(dev)
    W = []
    for _ in range(copies):
        b = torch.empty(wb, dtype=torch.uint8, device=dev)
        mgb.repack(fmt, src.data_ptr(), n, k, b.data_ptr(), stream.cuda_stream)
        W.append(b)
    del src
    x = torch.from_numpy(synthetic.activations(m, k)).to(dev)
    y = torch.empty((m, n), dtype=torch.float32, device=dev)
    ws_fn = mgb.qmatmul_min_workspace_bytes if args.min_workspace else mgb.qmatmul_workspace_bytes
    ws_bytes = ws_fn(fmt, m, n, k)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)

    def launch(i: int, s: int) -> None:
        mgb.qmatmul(fmt, W[i % copies].data_ptr(), n, k, x.data_ptr(), m, y.data_ptr(),
                    workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=s)

    if args.graph:
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            for i in range(copies):
                launch(i, cap.cuda_stream)
            with torch.cuda.graph(graph, stream=cap):
                for i in range(copies):
                    launch(i, torch.cuda.current_stream().cuda_stream)
        stream.wait_stream(cap)
        reps = max(1, -(-args.launches // copies))

        def run(count: int) -> None:
            for _ in range(count):
                graph.replay()
        launches = reps * copies
        warm = max(1, args.warmup)
        work = reps
    else:
        def run(count: int) -> None:
            for i in range(count):
                launch(i, stream.cuda_stream)
        launches = args.launches
        warm = args.warmup
        work = launches
    run(warm)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    h0 = time.perf_counter()
    t0.record(stream)
    run(work)
    t1.record(stream)
    h1 = time.perf_counter()
    torch.cuda.synchronize()
    h2 = time.perf_counter()
    us = t0.elapsed_time(t1) * 1e3 / launches
    assert mgb.take_device_error(0) == 0
    algo = wb + 4 * m * (n + k)
    print(json.dumps({"fmt": args.fmt, "m": m, "n": n, "k": k, "us_per_launch": us,
                      "weight_bytes": wb, "gbs": algo / (us * 1e-6) / 1e9,
                      "tflops": 2.0 * m * n * k / (us * 1e-6) / 1e12, "copies": copies,
                      "launches": launches, "graph": args.graph,
                      "host_enqueue_us": (h1 - h0) * 1e6 / launches,
                      "host_total_us": (h2 - h0) * 1e6 / launches,
                      "workspace_bytes": ws_bytes}), flush=True)


if __name__ == "__main__":
    main()
