#!/usr/bin/env python
"""Headline benchmark of the B200 packed-weight matmul Provider.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: Q4_K prefill GEMM, f32 activations
X[512, 4096] ~ N(0, 1) times Q4_K W[14336 x 4096] (random blocks with
f16 d, dmin ~ U(1e-3, 1e-2)), f32 output.  A step is one call of the path
over one batch.  Metric: TFLOP/s (2*M*N*K per step), whole job.

- value: device-resident inputs, the low-level C entry `mgb_qmatmul`
  (f32 -> bf16 activation pass + tcgen05 GEMM), CUDA events on the launching
  stream, inputs rotated over enough distinct sets to exceed 3x L2.
- e2e: the same metric through the Provider C ABI with host buffers:
  write_tensor from pinned memory (H2D), submit_kernel("matmul"),
  complete_kernel, read_tensor into pinned memory (D2H), every step.
- roofline: the GEMM kernel alone (`mgb_qmatmul_bf16`), FLOPs per launch over
  its event-timed average duration, against MEASURED_PEAKS.json's burst bf16.
- gemv: config 0 (Q4_K decode GEMV 1x4096 x 4096x4096) weight GB/s, as the
  second half of the BASELINE metric.
- formats: every format the Provider executes (Q4_K, Q5_K, Q6_K, Q8_0,
  IQ4_NL, Q4_0) at config 2's K=4096, N=14336: decode GEMV (M=1) weight GB/s and the
  prefill step (M=512) TFLOP/s, each over a CUDA graph of back-to-back
  launches on rotating weight copies (--no-formats skips it).
- stacks (one GPU): config 3, the Llama-3-8B decode stack (32 layers of
  Wq/Wk/Wv/Wo/gate/up/down, Q4_K) at M = 1, 16, 64, and config 4, the
  Llama-3-70B layers (80 layers) at M = 1 and 2048: one CUDA graph per pass
  over every layer's own weights; weight GB/s and TFLOP/s (--no-stacks skips).
  --tp-stacks adds the same passes under tensor parallelism (config 3 at M = 1, 16;
  config 4 at M = 1, 2048): fused calls with device epochs, one CUDA graph per pass.
- cpu_baseline: the reference's own CPU path (int8 activations, AVX2 kernels,
  persistent pool), restated in C (oracle/cpu_baseline.c), on a sample of
  the same workload, on every host core.
N > 1 (torchrun): tensor parallel along N (each rank holds 14336/N weight
rows); the kernels store every output column into every rank's y over NVLink
(CUDA IPC mappings) and a stream-ordered wait completes the step
(`tp.FusedShardedPackedMatmul`); strong scaling, max over ranks.  The NCCL
all-gather variant (`tp.gather_columns`) is timed beside it as
`tp_baseline_nccl`.  e2e at N > 1: pinned x -> device, the fused call, the
full y -> pinned host, on every rank.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import re
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
PKG = ROOT / "magnetar-provider-cpu_b200"
for _p in (ROOT, PKG):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

M, K, N = 512, 4096, 14336
GEMV_N = GEMV_K = 4096
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "Q4_K prefill GEMM TFLOP/s (X[512,4096] f32 x Q4_K W[14336x4096] -> f32)"
WORKLOAD = "config1: Q4_K prefill GEMM M=512 K=4096 N=14336 (Llama-3-8B FFN gate/up)"
GEMV_WORKLOAD = "config0: Q4_K decode GEMV x[1,4096] f32 x W[4096x4096] -> f32"
GEMV_METRIC = "Q4_K decode GEMV weight GB/s (config0: x[1,4096] x W[4096x4096])"


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            return json.loads(path.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


# DRAM traffic measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum of one launch)
# beside the algorithmic bytes of the same launch: the config-1 GEMM alone (bf16 x read,
# packed W read; its f32 y stayed in L2 under the capture) and the config-0 GEMV (packed W,
# f32 x and y).  The summaries and their commands are profiles/gemm_q4k_config1.md and
# profiles/gemv_q4k_config0.md.  A launch of another size (a tensor-parallel shard)
# reports the measured bytes scaled by its own algorithmic bytes: the traffic of these
# kernels grows in proportion to the weight rows they stream.
NCU_TRAFFIC = {
    "gemm_q4k_config1": {"dram_bytes": 38_770_176, "algorithmic_bytes": 33_030_144 + 4_194_304},
    "gemv_q4k_config0": {"dram_bytes": 9_493_760, "algorithmic_bytes": 9_469_952},
}


def scaled_traffic(name: str, algorithmic_bytes: float) -> dict:
    ref = NCU_TRAFFIC[name]
    return {"bytes_per_launch": ref["dram_bytes"] * algorithmic_bytes / ref["algorithmic_bytes"],
            "basis": f"ncu dram bytes of {name} ({ref['dram_bytes']} B per launch) scaled by "
                     f"this launch's algorithmic bytes ({algorithmic_bytes:.0f} / "
                     f"{ref['algorithmic_bytes']})"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(gpu_index)], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.flush()
        rows = []
        for line in pathlib.Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1])]
        sm_max = max((num(r[2]) or 0) for r in rows)
        loaded = [s for s in sm if s and s > 0.5 * sm_max] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": sm_max,
                "reasons": reasons, "samples": len(rows), "samples_under_load": len(loaded),
                "power_w_max": max((num(r[3]) or 0) for r in rows)}


# ---------------------------------------------------------------------------------------
# the reference arm: the reference's own CPU path on the host cores
# ---------------------------------------------------------------------------------------


def cpu_baseline(steps: int, warmup: int, budget_s: float = 20.0) -> dict:
    """Times the CPU port of the reference's default path (int8 activations,
    AVX2 Q4_K kernel, pool over all host threads) on a column sample of config 1,
    each call sized so that steps + warmup calls take about `budget_s`."""
    import numpy as np

    import synthetic
    from oracle import oracle

    threads = os.cpu_count() or 1
    x = synthetic.activations(M, K)
    full = synthetic.packed_weights(synthetic.Q4_K, N, K)
    ncols = 256
    cols = np.arange(ncols)
    w = synthetic.row_slice(synthetic.Q4_K, full, K, cols)
    t0 = time.perf_counter()
    oracle.baseline_packed_matmul(synthetic.Q4_K, w, ncols, K, x, int8=True, threads=threads)
    one = time.perf_counter() - t0
    target = max(0.02, budget_s / max(1, steps + warmup))
    ncols = int(min(N, max(64, ncols * target / max(one, 1e-6))) // 64 * 64) or 64
    w = synthetic.row_slice(synthetic.Q4_K, full, K, np.arange(ncols))
    for _ in range(warmup):
        oracle.baseline_packed_matmul(synthetic.Q4_K, w, ncols, K, x, int8=True, threads=threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.baseline_packed_matmul(synthetic.Q4_K, w, ncols, K, x, int8=True, threads=threads)
    dt = (time.perf_counter() - t0) / steps
    flops = 2.0 * M * ncols * K
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"M={M} K={K}, first {ncols} of {N} output columns per call, "
                      f"{steps} timed calls of {dt * 1e3:.2f} ms after {warmup} warm-up",
            "ms_per_call": dt * 1e3}


def cpu_gemv_baseline(repeats: int = 10) -> dict:
    """Config 0 on the CPU port of the reference's default path (M = 1, Q4_K
    4096 x 4096, int8 activations, AVX2 kernel, pool over all host threads),
    timed as the reference's own decode diagnostic times it
    (`packed_matmul_bandwidth`, src/native/tests.rs:333-376: one warm-up call,
    then the mean of `repeats` calls on the same weight; weight GB/s)."""
    from oracle import oracle

    import synthetic

    threads = os.cpu_count() or 1
    w = synthetic.packed_weights(synthetic.Q4_K, GEMV_N, GEMV_K)
    x = synthetic.activations(1, GEMV_K)
    oracle.baseline_packed_matmul(synthetic.Q4_K, w, GEMV_N, GEMV_K, x, int8=True, threads=threads)
    t0 = time.perf_counter()
    for _ in range(repeats):
        oracle.baseline_packed_matmul(synthetic.Q4_K, w, GEMV_N, GEMV_K, x, int8=True,
                                      threads=threads)
    dt = (time.perf_counter() - t0) / repeats
    algo = w.size + GEMV_K * 4 + GEMV_N * 4
    return {"value": algo / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"config 0 in full (x[1,{GEMV_K}] x Q4_K W[{GEMV_N}x{GEMV_K}]), one warm-up "
                      f"then the mean of {repeats} calls on the same weight "
                      "(the reference's packed_matmul_bandwidth method)",
            "us_per_call": dt * 1e6}


def config_dict() -> dict:
    """The workload, identical in both arms (how each arm runs it is in `details`)."""
    return {"workload": WORKLOAD, "m": M, "k": K, "n": N, "format": "Q4_K",
            "gemv_workload": GEMV_WORKLOAD}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # under torchrun only rank 0 runs the CPU arm
    steps, warmup = args.steps, args.warmup
    cb = cpu_baseline(steps, warmup, budget_s=60.0)
    gv = cpu_gemv_baseline()
    line = {"metric": METRIC, "value": cb["value"], "unit": "TFLOP/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": warmup, "ms_per_step": cb["ms_per_call"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8 x u4 dots, f32 accumulate", "data": "synthetic", "impl": "reference",
            "config": config_dict(),
            "details": {"parallelism": f"{cb['cores']} host threads (the reference's pool)",
                        "step": "C port of the reference's packed_matmul: quantize_rows + "
                                "columns_q4k_avx2 over the pool partition of "
                                "src/native/mod.rs:135-150"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "gemv": {"metric": GEMV_METRIC, "value": gv["value"], "unit": "GB/s",
                     "cpu_baseline": gv}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------------------


def run_b200(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist

    import magnetar_b200 as mgb
    import synthetic
    import tp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    lo, hi = tp.shard_bounds(N, world, rank)
    n_loc = hi - lo
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    fmt = mgb.Q4_K

    # weights: this rank's stored rows, in the device layout, rotated over R copies
    full = synthetic.packed_weights(fmt, N, K)
    w_loc = np.array(tp.shard_packed(fmt, full, N, K, world, rank))
    del full
    w_bytes = mgb.packed_bytes(fmt, n_loc, K)
    set_bytes = w_bytes + M * K * 4 + M * n_loc * 4
    R = max(2, -(-3 * L2_BYTES // set_bytes))
    ggml = torch.from_numpy(w_loc).to(dev)
    W = []
    for _ in range(R):
        buf = torch.empty(w_bytes, dtype=torch.uint8, device=dev)
        mgb.repack(fmt, ggml.data_ptr(), n_loc, K, buf.data_ptr(), sp)
        W.append(buf)
    del ggml
    x_host = synthetic.activations(M, K)
    X = [torch.from_numpy(x_host).to(dev) for _ in range(R)]
    Y = [torch.empty((M, n_loc), dtype=torch.float32, device=dev) for _ in range(R)]
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, M, n_loc, K)
    WS = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)

    op = None
    if world > 1:
        op = tp.FusedShardedPackedMatmul(fmt, w_loc, N, K, world, rank, max_m=M, device=dev,
                                         device_epochs=True)

    def step(i: int) -> None:
        s = i % R
        if op is not None:  # fused all-gather: [M, N] on every rank
            op.weight = W[s]
            op(X[s])
            return
        mgb.qmatmul(fmt, W[s].data_ptr(), n_loc, K, X[s].data_ptr(), M, Y[s].data_ptr(),
                    workspace_ptr=WS.data_ptr(), workspace_bytes=ws_bytes, stream=sp)

    # Under tensor parallelism the steps run as CUDA graphs of fused calls (device
    # epochs), so the host's per-call work (ctypes, the output description) is out of
    # the device's way: one graph of the W warm-up steps, one of the K timed steps,
    # captured in that order and each replayed once, so the calls' y buffers keep
    # alternating from one graph into the next.
    graphs = {}
    if op is not None:
        step(0)  # eager: workspace allocated, kernels configured
        torch.cuda.synchronize()
        cap = torch.cuda.Stream(device=dev)
        cap.wait_stream(stream)
        for name, count in (("warm", args.warmup), ("timed", args.steps)):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(g, stream=cap):
                    for i in range(count):
                        step(i)
            graphs[name] = g
        stream.wait_stream(cap)
        torch.cuda.synchronize()

    def step_nccl(i: int) -> None:
        s = i % R
        mgb.qmatmul(fmt, W[s].data_ptr(), n_loc, K, X[s].data_ptr(), M, Y[s].data_ptr(),
                    workspace_ptr=WS.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
        tp.gather_columns(Y[s])  # [M, N] on every rank

    def timed(fn, steps: int, warmup: int, whole=None) -> float:
        """Device time of `steps` calls of fn after `warmup` untimed ones, max over
        ranks; `whole` = (warm-up graph, timed graph) replaces the calls."""
        if whole is not None:
            whole[0].replay()
        for i in range(warmup if whole is None else 0):
            fn(i)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        if whole is not None:
            whole[1].replay()
        for i in range(steps if whole is None else 0):
            fn(i)
        t1.record(stream)
        torch.cuda.synchronize()
        ms = t0.elapsed_time(t1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    sampler = ClockSampler(visible[local] if local < len(visible) else str(local))
    total_ms = timed(step, args.steps, args.warmup,
                     (graphs["warm"], graphs["timed"]) if graphs else None)
    if op is not None:
        assert mgb.take_device_error(local) == 0, "a tensor-parallel wait gave up"
        graphs.clear()
    ms_step = total_ms / args.steps
    flops = 2.0 * M * N * K
    value = flops / (ms_step * 1e-3) / 1e12
    nccl = None
    if world > 1:
        nccl_ms = timed(step_nccl, args.steps, args.warmup) / args.steps
        nccl = {"ms_per_step": nccl_ms, "value": flops / (nccl_ms * 1e-3) / 1e12,
                "unit": "TFLOP/s", "step": "mgb_qmatmul into [M, N/G] + NCCL "
                                           "all_gather_into_tensor + interleave"}

    # roofline: the GEMM kernel alone on bf16 activations
    XB = [x.to(torch.bfloat16) for x in X]

    def gemm_only(i: int) -> None:
        s = i % R
        mgb.qmatmul_bf16(fmt, W[s].data_ptr(), n_loc, K, XB[s].data_ptr(), M, Y[s].data_ptr(),
                         stream=sp)

    gemm_ms = timed(gemm_only, args.steps, args.warmup) / args.steps
    clocks = sampler.stop()
    pk, pk_kind = peaks()
    achieved = 2.0 * M * n_loc * K / (gemm_ms * 1e-3) / 1e12
    tr = scaled_traffic("gemm_q4k_config1", w_bytes + M * K * 2)
    roofline = {"bound": "tensor", "kernel": "mgb_gemm_kernel<Q4_K> (tcgen05, bf16 x bf16 -> f32)",
                "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved / pk["bf16_tflops"], "peak_kind": f"{pk_kind} burst bf16",
                "traffic": tr["bytes_per_launch"], "traffic_basis": tr["basis"],
                "ms_per_launch": gemm_ms, "flops_per_launch": 2.0 * M * n_loc * K}

    # e2e with pinned host buffers: through the Provider's C ABI on one GPU,
    # through the fused tensor-parallel call on several
    xh = torch.from_numpy(x_host).pin_memory()
    prov = None
    if op is None:
        prov = mgb.B200Provider(device=local)
        assert prov.write_packed_weight_tensor("w", fmt, n_loc, K, True, w_loc) == "Stored"
        # two requests in flight, as a serving runtime keeps them: each host
        # thread owns its x/y resources and pinned buffers, so one step's
        # download overlaps the next step's upload and kernel
        xhs = [xh, torch.from_numpy(x_host).pin_memory()]
        yhs = [torch.empty((M, n_loc), dtype=torch.float32).pin_memory() for _ in range(2)]

        def e2e_step(i: int) -> None:
            s = i % 2
            prov.write_tensor_ptr(f"x{s}", (M, K), xhs[s].data_ptr())
            h = prov.submit_kernel("matmul", [f"x{s}", "w"], f"y{s}")
            r = prov.complete_kernel(h)
            if not r.ok:
                raise RuntimeError(r.reason)
            prov.read_tensor_into(f"y{s}", yhs[s].data_ptr(), M * n_loc)
    else:
        op.weight = W[0]
        yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
        xd = torch.empty((M, K), dtype=torch.float32, device=dev)

        def e2e_step(_i: int) -> None:
            xd.copy_(xh, non_blocking=True)
            yh.copy_(op(xd), non_blocking=True)
            stream.synchronize()

    e2e_steps = max(4, min(args.steps, 50)) // 2 * 2
    for i in range(max(4, args.warmup)):
        e2e_step(i)
    serial_s = None
    if prov is not None:
        t0 = time.perf_counter()  # one thread: every call waits for the one before
        for i in range(e2e_steps):
            e2e_step(i)
        serial_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    if prov is not None:
        errors: list[BaseException] = []

        def lane(s: int) -> None:
            try:
                for i in range(s, e2e_steps, 2):
                    e2e_step(i)
            except BaseException as ex:  # re-raised below
                errors.append(ex)

        lanes = [threading.Thread(target=lane, args=(s,)) for s in range(2)]
        for t in lanes:
            t.start()
        for t in lanes:
            t.join()
        if errors:
            raise errors[0]
    else:
        for i in range(e2e_steps):
            e2e_step(i)
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    if prov is not None:
        prov.close()
        if not torch.equal(yhs[0], yhs[1]):
            raise RuntimeError("the two e2e lanes returned different outputs for the same input")
        path = ("mgb_write_tensor (pinned) -> mgb_submit_kernel(matmul) -> mgb_complete_kernel -> "
                "mgb_read_tensor (pinned), on two host threads with their own x/y resources "
                "(two steps in flight: one step's download overlaps the next one's upload and "
                "kernel); wall clock")
        d2h = M * N * 4
    else:
        path = ("pinned x -> device, tp.FusedShardedPackedMatmul (mgb_qmatmul_tp + mgb_tp_wait), "
                "full y [M, N] -> pinned host on every rank; wall clock")
        d2h = M * N * 4 * world
    e2e = {"value": flops / e2e_s / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": M * K * 4 * world,
           "d2h_bytes_per_step": d2h, "ms_per_step": e2e_s * 1e3, "steps": e2e_steps,
           "path": path, "timing": "wall clock per rank, max over ranks"}
    if serial_s is not None:
        e2e["one_thread_ms_per_step"] = serial_s * 1e3

    def graph_ms(gfmt: int, m: int, n: int, k: int, min_launches: int) -> tuple[float, int, int, int]:
        """Device time per `mgb_qmatmul` (x [m, k] f32 -> y [m, n] f32) over
        replays of one CUDA graph of back-to-back launches, one per weight copy,
        with enough copies to exceed 3x L2.  Returns (ms, weight bytes,
        copies, replays)."""
        gw = synthetic.packed_weights(gfmt, n, k)
        gb = mgb.packed_bytes(gfmt, n, k)
        copies = max(2, -(-3 * L2_BYTES // gb))
        src = torch.from_numpy(gw).to(dev)
        GW = []
        for _ in range(copies):
            b = torch.empty(gb, dtype=torch.uint8, device=dev)
            mgb.repack(gfmt, src.data_ptr(), n, k, b.data_ptr(), sp)
            GW.append(b)
        del src
        gx = torch.from_numpy(synthetic.activations(m, k)).to(dev)
        gy = torch.empty((m, n), dtype=torch.float32, device=dev)
        gws_bytes = mgb.qmatmul_workspace_bytes(gfmt, m, n, k)
        gws = torch.empty(max(gws_bytes, 16), dtype=torch.uint8, device=dev)
        cap = torch.cuda.Stream(device=dev)
        graph = torch.cuda.CUDAGraph()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            for i in range(copies):  # warm the launch path outside capture
                mgb.qmatmul(gfmt, GW[i].data_ptr(), n, k, gx.data_ptr(), m, gy.data_ptr(),
                            workspace_ptr=gws.data_ptr(), workspace_bytes=gws_bytes,
                            stream=cap.cuda_stream)
            with torch.cuda.graph(graph, stream=cap):
                for i in range(copies):
                    mgb.qmatmul(gfmt, GW[i].data_ptr(), n, k, gx.data_ptr(), m, gy.data_ptr(),
                                workspace_ptr=gws.data_ptr(), workspace_bytes=gws_bytes,
                                stream=torch.cuda.current_stream().cuda_stream)
        stream.wait_stream(cap)
        reps = max(3, -(-min_launches // copies))
        ms = timed_local(lambda _i: graph.replay(), reps, 3) / (reps * copies)
        del graph
        return ms, gb, copies, reps

    def timed_local(fn, steps: int, warmup: int) -> float:
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(steps):
            fn(i)
        t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1)

    # second half of the metric: config 0 decode GEMV weight GB/s (rank 0's GPU)
    gemv = None
    formats = None
    if rank == 0:
        g_ms, gb, RV, reps = graph_ms(fmt, 1, GEMV_N, GEMV_K, max(args.steps, 200))
        algo = gb + GEMV_K * 4 + GEMV_N * 4
        gbs = algo / (g_ms * 1e-3) / 1e9
        tr = scaled_traffic("gemv_q4k_config0", algo)
        gemv = {"metric": GEMV_METRIC, "value": gbs, "unit": "GB/s", "us_per_launch": g_ms * 1e3,
                "algorithmic_bytes": algo,
                "roofline": {"bound": "hbm", "kernel": "mgb_gemv_staged_kernel<Q4_K>",
                             "achieved": gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": gbs / pk["hbm_gbs"], "peak_kind": f"{pk_kind} HBM copy",
                             "traffic": tr["bytes_per_launch"], "traffic_basis": tr["basis"]},
                "l2": f"{RV} rotating weight copies ({RV * gb / 1e6:.0f} MB > 3x L2)",
                "timing": f"CUDA events around {reps} replays of a CUDA graph of {RV} "
                          "back-to-back launches (programmatic dependent launches)",
                "cpu_baseline": None}
        # the same GEMV at config 4's widest decode projection (Llama-3-70B
        # gate/up: x[1, 8192] x W[28672 x 8192]), where the weight stream, not
        # the launch floor, sets the time
        l_ms, lb, LRV, lreps = graph_ms(fmt, 1, 28672, 8192, 60)
        l_gbs = (lb + 8192 * 4 + 28672 * 4) / (l_ms * 1e-3) / 1e9
        gemv["large"] = {"shape": "x[1,8192] x Q4_K W[28672x8192] (config 4 gate/up)",
                         "us_per_launch": l_ms * 1e3, "gbs": l_gbs,
                         "frac_hbm": l_gbs / pk["hbm_gbs"],
                         "timing": f"{lreps} replays of a graph of {LRV} launches over "
                                   f"{LRV} weight copies"}

        # every format the Provider executes, at config 2's shape (K = 4096,
        # N = 14336): decode GEMV (M = 1) weight GB/s and prefill step (M = 512,
        # activation cast + tcgen05 GEMM) TFLOP/s, same graph timing
        if not args.no_formats:
            formats = {}
            for name, f in (("q4_k", mgb.Q4_K), ("q5_k", mgb.Q5_K), ("q6_k", mgb.Q6_K),
                            ("q8_0", mgb.Q8_0), ("iq4_nl", mgb.IQ4_NL), ("q4_0", mgb.Q4_0)):
                v_ms, vb, _, _ = graph_ms(f, 1, N, K, 100)
                v_gbs = (vb + K * 4 + N * 4) / (v_ms * 1e-3) / 1e9
                p_ms, _, _, _ = graph_ms(f, M, N, K, 40)
                formats[name] = {"gemv_us": v_ms * 1e3, "gemv_gbs": v_gbs,
                                 "gemv_frac_hbm": v_gbs / pk["hbm_gbs"],
                                 "prefill_us": p_ms * 1e3,
                                 "prefill_tflops": 2.0 * M * N * K / (p_ms * 1e-3) / 1e12,
                                 "device_bytes": vb}

    def stack(shapes: list[tuple[int, int]], layers: int, m: int) -> dict:
        """Configs 3 and 4: `layers` layers of Q4_K projections, `shapes` =
        (n, k) per projection in order, one `mgb_qmatmul` each (M activation
        rows), captured as one CUDA graph; every layer holds its own device
        copy of each weight (one host-generated matrix per shape, repacked,
        then copied on the device), so a pass streams all layers' weights."""
        per_shape = {}
        for (n, k) in sorted(set(shapes)):
            src = torch.from_numpy(synthetic.packed_weights(fmt, n, k, seed=n + k)).to(dev)
            b = torch.empty(mgb.packed_bytes(fmt, n, k), dtype=torch.uint8, device=dev)
            mgb.repack(fmt, src.data_ptr(), n, k, b.data_ptr(), sp)
            per_shape[(n, k)] = b
            del src
        layer_w = [[per_shape[s].clone() for s in shapes] for _ in range(layers)]
        del per_shape
        xs = {k: torch.from_numpy(synthetic.activations(m, k, seed=k)).to(dev)
              for k in sorted({k for _, k in shapes})}
        ys = {n: torch.empty((m, n), dtype=torch.float32, device=dev)
              for n in sorted({n for n, _ in shapes})}
        ws_bytes = max(mgb.qmatmul_workspace_bytes(fmt, m, n, k) for n, k in shapes)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)

        def one_pass(s: int) -> None:
            for lw in layer_w:
                for (n, k), w in zip(shapes, lw):
                    mgb.qmatmul(fmt, w.data_ptr(), n, k, xs[k].data_ptr(), m, ys[n].data_ptr(),
                                workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=s)

        cap = torch.cuda.Stream(device=dev)
        graph = torch.cuda.CUDAGraph()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            one_pass(cap.cuda_stream)  # warm the launch path outside capture
            with torch.cuda.graph(graph, stream=cap):
                one_pass(torch.cuda.current_stream().cuda_stream)
        stream.wait_stream(cap)
        probe = timed_local(lambda _i: graph.replay(), 1, 1)
        reps = int(max(2, min(50, 1000.0 / max(probe, 1e-3))))  # about a second
        pass_ms = timed_local(lambda _i: graph.replay(), reps, 2) / reps
        del graph
        wbytes = layers * sum(mgb.packed_bytes(fmt, n, k) for n, k in shapes)
        flops = 2.0 * m * layers * sum(n * k for n, k in shapes)
        gbs = wbytes / (pass_ms * 1e-3) / 1e9
        tfl = flops / (pass_ms * 1e-3) / 1e12
        out = {"m": m, "ms_per_pass": pass_ms, "tokens_per_s": m / (pass_ms * 1e-3),
               "weight_bytes": wbytes, "weight_gbs": gbs, "frac_hbm": gbs / pk["hbm_gbs"],
               "tflops": tfl, "frac_bf16": tfl / pk["bf16_tflops_sustained"],
               "launches_per_pass": layers * len(shapes), "replays": reps}
        del layer_w, xs, ys, ws
        torch.cuda.empty_cache()
        return out

    # configs 3 and 4 on one GPU: whole projection stacks, one graph per pass
    stacks = None
    if rank == 0 and world == 1 and not args.no_stacks:
        l8 = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096),
              (14336, 4096), (4096, 14336)]
        l70 = [(8192, 8192), (1024, 8192), (1024, 8192), (8192, 8192), (28672, 8192),
               (28672, 8192), (8192, 28672)]
        stacks = {
            "config3": {"workload": "Llama-3-8B decode stack: 32 layers x {Wq, Wk, Wv, Wo, "
                                    "gate, up, down}, Q4_K, random weights",
                        "passes": [stack(l8, 32, mm) for mm in (1, 16, 64)]},
            "config4": {"workload": "Llama-3-70B layers: 80 layers x {Wq, Wk, Wv, Wo, gate, "
                                    "up, down}, Q4_K, random weights",
                        "passes": [stack(l70, 80, mm) for mm in (1, 2048)]},
            "peaks": "frac_hbm of the measured HBM copy, frac_bf16 of the measured "
                     "sustained bf16 (a pass is a long step)",
            "timing": "CUDA events around replays of one CUDA graph holding one pass "
                      "(every projection of every layer once; weights far above L2)"}

    def tp_stack(shapes: list[tuple[int, int]], layers: int, m: int) -> dict:
        """A stack pass under tensor parallelism: every projection one fused
        call on this rank's N/G stored rows (columns stored into every rank's
        y; each call waits, inside its first kernel, for the call before it on
        every rank), with device epochs, the whole pass captured as one CUDA
        graph.  One fused op per distinct shape, its
        weight swapped for each layer's own copy (every shape is called an
        even number of times per pass, so its two y buffers keep alternating
        across replays)."""
        ops = {}
        graph = None
        try:
            for (n, k) in sorted(set(shapes)):
                full = synthetic.packed_weights(fmt, n, k, seed=n + k)
                ops[(n, k)] = tp.FusedShardedPackedMatmul(
                    fmt, tp.shard_packed(fmt, full, n, k, world, rank), n, k, world, rank,
                    max_m=m, device=dev, device_epochs=True)
                del full
            layer_w = [[ops[s].weight.clone() for s in shapes] for _ in range(layers)]
            xs = {k: torch.from_numpy(synthetic.activations(m, k, seed=k)).to(dev)
                  for k in sorted({k for _, k in shapes})}

            def one_pass() -> None:
                # each call waits for the call before it (the previous pass's
                # last, for the first) inside its own first kernel, as a model
                # whose next projection reads the gathered y would; only the
                # pass's last call is followed by a wait of its own
                prev = ops[shapes[-1]]
                for li, lw in enumerate(layer_w):
                    for si, (s, w) in enumerate(zip(shapes, lw)):
                        last = li == len(layer_w) - 1 and si == len(shapes) - 1
                        ops[s].weight = w
                        ops[s](xs[s[1]], after=prev, wait=last)
                        prev = ops[s]

            one_pass()  # eager: workspaces allocated, kernels configured
            torch.cuda.synchronize()
            cap = torch.cuda.Stream(device=dev)
            cap.wait_stream(stream)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.stream(cap):
                with torch.cuda.graph(graph, stream=cap):
                    one_pass()
            stream.wait_stream(cap)
            probe = timed(lambda _i: graph.replay(), 1, 1)
            reps = int(max(2, min(50, 1000.0 / max(probe, 1e-3))))
            pass_ms = timed(lambda _i: graph.replay(), reps, 2) / reps
            assert mgb.take_device_error(local) == 0, "a tensor-parallel wait gave up"
            wbytes = layers * sum(mgb.packed_bytes(fmt, n, k) for n, k in shapes)
            flops = 2.0 * m * layers * sum(n * k for n, k in shapes)
            gbs = wbytes / (pass_ms * 1e-3) / 1e9
            tfl = flops / (pass_ms * 1e-3) / 1e12
            return {"m": m, "ms_per_pass": pass_ms, "tokens_per_s": m / (pass_ms * 1e-3),
                    "weight_gbs": gbs, "weight_gbs_per_gpu": gbs / world,
                    "frac_hbm_per_gpu": gbs / world / pk["hbm_gbs"], "tflops": tfl,
                    "frac_bf16_per_gpu": tfl / world / pk["bf16_tflops_sustained"],
                    # per call: (activation cast +) GEMM or GEMV, then the publish
                    # kernel; one wait kernel after the pass's last call
                    "launches_per_pass": (3 if m > 2 else 2) * layers * len(shapes) + 1,
                    "replays": reps}
        finally:
            del graph
            for op in ops.values():
                op.close()
            torch.cuda.empty_cache()

    tp_stacks = None
    if args.tp_stacks or (world > 1 and not args.no_tp_stacks):
        l8 = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096),
              (14336, 4096), (4096, 14336)]
        l70 = [(8192, 8192), (1024, 8192), (1024, 8192), (8192, 8192), (28672, 8192),
               (28672, 8192), (8192, 28672)]
        tp_stacks = {
            "config3": {"workload": f"Llama-3-8B decode stack, tp{world}",
                        "passes": [tp_stack(l8, 32, mm) for mm in (1, 16)]},
            "config4": {"workload": f"Llama-3-70B layers, tp{world}",
                        "passes": [tp_stack(l70, 80, mm) for mm in (1, 2048)]},
            "timing": "CUDA events around replays of one CUDA graph per pass (fused calls "
                      "with device epochs), max over ranks"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(steps=10, warmup=1)
        if gemv is not None:
            gemv["cpu_baseline"] = cpu_gemv_baseline()

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16 operands, f32 accumulate", "data": "synthetic",
                "config": config_dict(),
                "details": {"n_per_rank": n_loc, "parallelism": f"tp{world}",
                            "l2": f"{R} rotating input sets of {set_bytes / 1e6:.0f} MB "
                                  f"({R * set_bytes / 1e6:.0f} MB > 3x 126 MB L2)",
                            "step": "mgb_qmatmul: f32->bf16 activation pass + tcgen05 GEMM"
                                    + (" storing every column into every rank's y over NVLink "
                                       "+ stream-ordered wait for all ranks (mgb_qmatmul_tp, "
                                       "mgb_tp_wait), device epochs; the warm-up and timed "
                                       "steps each one CUDA graph" if world > 1 else "")},
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
                "gpu_launches": (4 if world > 1 else 2) * args.steps, "clocks": clocks,
                "gemv": gemv, "formats": formats, "stacks": stacks, "tp_stacks": tp_stacks,
                "tp_baseline_nccl": nccl}
        print(json.dumps(line), flush=True)
    if op is not None:
        op.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-formats", action="store_true", help="skip the per-format table")
    ap.add_argument("--tp-stacks", action="store_true",
                    help="also time the config-3/4 stacks under tensor parallelism at N = 1 "
                         "(CUDA graphs of fused calls; on by default at N > 1)")
    ap.add_argument("--no-tp-stacks", action="store_true",
                    help="skip the tensor-parallel config-3/4 stacks at N > 1")
    ap.add_argument("--no-stacks", action="store_true",
                    help="skip the config-3/4 projection stacks (one GPU)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
