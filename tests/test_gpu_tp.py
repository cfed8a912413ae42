"""GPU parity of the fused tensor-parallel path (`mgb_qmatmul_tp`, `mgb_tp_wait`).

Each rank's kernels store its columns into every rank's y and publish the
call's epoch.  On one GPU the ranks are emulated: rank 0's and rank 1's calls
run one after the other on the same stream with two local y buffers and two
sets of synchronisation words, and the waits run after both calls have
finished (no kernel waits on another kernel that may still be running on
the same GPU).  With two GPUs, two processes run the real path over NVLink.

Every output column is computed by the same kernels as a plain call on the
rank's shard (the split is by whole stored rows, `packed_matmul`,
src/native/mod.rs:135-150), so the gathered y must equal the plain
`mgb_qmatmul` of every shard side by side bit for bit (with the same
workspace, so the same split-K choice), and the oracle within the kernels'
tolerances.
"""

from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import magnetar_b200 as mgb
import synthetic
import tp

pytestmark = pytest.mark.gpu

GEMV_TOL, GEMM_TOL = 1e-3, 5e-3


@pytest.fixture(scope="module")
def torch_cuda(cuda_device):
    import torch

    torch.cuda.set_device(cuda_device)
    return torch


def _device_layout(torch, fmt, ggml, rows, cols):
    src = torch.from_numpy(np.ascontiguousarray(ggml)).cuda()
    out = torch.empty(mgb.packed_bytes(fmt, rows, cols), dtype=torch.uint8, device="cuda")
    mgb.repack(fmt, src.data_ptr(), rows, cols, out.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
    return out


def _plain_shards(torch, fmt, w, n, k, xd, world=1):
    """The plain `mgb_qmatmul` of each of `world` shards, side by side, each
    with its preferred workspace as the tensor-parallel calls get it (a split-K
    choice depends on the shard's width, so the shard is the unit that matches
    bit for bit)."""
    m = xd.shape[0]
    n_loc = n // world
    cols = []
    for r in range(world):
        wd = _device_layout(torch, fmt, tp.shard_packed(fmt, w, n, k, world, r), n_loc, k)
        y = torch.full((m, n_loc), float("nan"), dtype=torch.float32, device="cuda")
        ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n_loc, k)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
        mgb.qmatmul(fmt, wd.data_ptr(), n_loc, k, xd.data_ptr(), m, y.data_ptr(),
                    workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes,
                    stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        cols.append(y.cpu().numpy())
    return np.concatenate(cols, axis=1)


CASES = [
    # fmt, n, k, m: GEMV (one and two rows), the GEMM, the two-launch GEMV
    # (k > 8192), the direct-load GEMV (k % 256 != 0)
    (synthetic.Q4_K, 512, 1024, 1),
    (synthetic.Q4_K, 512, 1024, 2),
    (synthetic.Q4_K, 512, 1024, 5),
    (synthetic.Q4_K, 1024, 2048, 130),
    (synthetic.Q8_0, 256, 512, 3),
    (synthetic.IQ4_NL, 256, 512, 2),
    (synthetic.Q4_0, 256, 512, 64),
    (synthetic.Q4_K, 256, 16384, 2),
    (synthetic.Q8_0, 128, 96, 2),
    (synthetic.Q8_0, 64, 8224, 2),
    (synthetic.Q6_K, 512, 1024, 1),
    (synthetic.Q6_K, 512, 1024, 96),
    (synthetic.Q6_K, 128, 32768, 2),
    (synthetic.Q5_K, 512, 1024, 2),
    (synthetic.Q5_K, 512, 1024, 96),
    (synthetic.Q5_K, 128, 32768, 1),
]


@pytest.mark.parametrize("fmt,n,k,m", CASES)
def test_emulated_two_ranks_gather_every_column(torch_cuda, oracle, fmt, n, k, m):
    torch = torch_cuda
    world = 2
    w = synthetic.packed_weights(fmt, n, k, seed=21)
    x = synthetic.activations(m, k, seed=22)
    xd = torch.from_numpy(x).cuda()
    shards = [_device_layout(torch, fmt, tp.shard_packed(fmt, w, n, k, world, r), n // world, k)
              for r in range(world)]
    ys = [torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") for _ in range(world)]
    sync = [mgb.device_alloc(mgb.TP_SYNC_BYTES) for _ in range(world)]
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n // world, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    try:
        for epoch in (1, 2, 3):  # the reserved words stay zero, the done words advance
            for r in range(world):
                out = mgb.tp_out([y.data_ptr() for y in ys], sync,
                                 sync[r] + mgb.TP_COUNTER_OFFSET, ldy=n, col0=r * (n // world),
                                 epoch=epoch, rank=r)
                mgb.qmatmul_tp(fmt, shards[r].data_ptr(), n // world, k, xd.data_ptr(), m, out,
                               workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
            for r in range(world):
                mgb.tp_wait(sync[r], world, epoch, 2000, sp)
            torch.cuda.synchronize()
            assert mgb.take_device_error(torch.cuda.current_device()) == 0
            for r in range(world):
                words = torch.as_tensor(tp._DeviceArray(sync[r], (mgb.TP_SYNC_BYTES // 4,)),
                                        device="cuda").view(torch.int32).cpu().numpy()
                assert list(words[:world]) == [epoch] * world
                assert words[mgb.TP_COUNTER_OFFSET // 4] == 0
        got = [y.cpu().numpy() for y in ys]
    finally:
        for p in sync:
            mgb.device_free(p)
    np.testing.assert_array_equal(got[0], got[1])
    np.testing.assert_array_equal(got[0], _plain_shards(torch, fmt, w, n, k, xd, world))
    oracle.assert_close(got[0], oracle.packed_matmul(fmt, w, n, k, x),
                        GEMV_TOL if m <= 2 else GEMM_TOL, f"tp fmt {fmt} m {m}")


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("fmt,n,k,m", [(synthetic.Q4_K, 512, 1024, 1),
                                       (synthetic.Q4_K, 512, 1024, 2),
                                       (synthetic.Q4_K, 512, 1024, 64),
                                       (synthetic.Q4_K, 1024, 2048, 130),
                                       (synthetic.Q6_K, 512, 1024, 96)])
def test_emulated_four_and_eight_ranks(torch_cuda, oracle, world, fmt, n, k, m):
    """The scaling run's group sizes: every rank stores into all 4 or 8 ranks'
    y and publishes into all of their done words (the eight-rank case fills
    every slot of the output description).  Ranks emulated one after the
    other on one GPU."""
    torch = torch_cuda
    w = synthetic.packed_weights(fmt, n, k, seed=24)
    x = synthetic.activations(m, k, seed=25)
    xd = torch.from_numpy(x).cuda()
    n_loc = n // world
    shards = [_device_layout(torch, fmt, tp.shard_packed(fmt, w, n, k, world, r), n_loc, k)
              for r in range(world)]
    ys = [torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") for _ in range(world)]
    sync = [mgb.device_alloc(mgb.TP_SYNC_BYTES) for _ in range(world)]
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n_loc, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    try:
        for epoch in (1, 2):
            for r in range(world):
                out = mgb.tp_out([y.data_ptr() for y in ys], sync,
                                 sync[r] + mgb.TP_COUNTER_OFFSET, ldy=n, col0=r * n_loc,
                                 epoch=epoch, rank=r)
                mgb.qmatmul_tp(fmt, shards[r].data_ptr(), n_loc, k, xd.data_ptr(), m, out,
                               workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
            for r in range(world):
                mgb.tp_wait(sync[r], world, epoch, 2000, sp)
            torch.cuda.synchronize()
            assert mgb.take_device_error(torch.cuda.current_device()) == 0
            for r in range(world):
                words = torch.as_tensor(tp._DeviceArray(sync[r], (mgb.TP_SYNC_BYTES // 4,)),
                                        device="cuda").view(torch.int32).cpu().numpy()
                assert list(words[:world]) == [epoch] * world
        got = [y.cpu().numpy() for y in ys]
    finally:
        for q in sync:
            mgb.device_free(q)
    ref = _plain_shards(torch, fmt, w, n, k, xd, world)
    for r in range(world):
        np.testing.assert_array_equal(got[r], ref)
    oracle.assert_close(got[0], oracle.packed_matmul(fmt, w, n, k, x),
                        GEMV_TOL if m <= 2 else GEMM_TOL, f"tp{world} fmt {fmt} m {m}")


@pytest.mark.parametrize("fmt,n,k,m", [(synthetic.Q4_K, 512, 1024, 64),
                                       (synthetic.Q4_K, 512, 1024, 1),
                                       (synthetic.Q6_K, 256, 16384, 2)])
def test_emulated_two_ranks_device_epochs_replay_in_a_graph(torch_cuda, fmt, n, k, m):
    """Device epochs (epoch 0): each rank's kernels publish its epoch word + 1
    and advance the word to it, so the two ranks' calls and waits captured
    in one CUDA graph publish fresh epochs on every replay.  Ranks are emulated
    one after the other on one GPU, as above; every replay's gathered y equals
    the unsharded call on that replay's activations."""
    torch = torch_cuda
    world = 2
    w = synthetic.packed_weights(fmt, n, k, seed=23)
    shards = [_device_layout(torch, fmt, tp.shard_packed(fmt, w, n, k, world, r), n // world, k)
              for r in range(world)]
    x = torch.zeros((m, k), dtype=torch.float32, device="cuda")
    ys = [torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda") for _ in range(world)]
    sync = [mgb.device_alloc(mgb.TP_SYNC_BYTES) for _ in range(world)]
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n // world, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")

    def one_pass(sp):
        for r in range(world):
            out = mgb.tp_out([y.data_ptr() for y in ys], sync, sync[r] + mgb.TP_COUNTER_OFFSET,
                             ldy=n, col0=r * (n // world), epoch=0, rank=r)
            mgb.qmatmul_tp(fmt, shards[r].data_ptr(), n // world, k, x.data_ptr(), m, out,
                           workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
        for r in range(world):
            mgb.tp_wait(sync[r], world, 0, 2000, sp)

    def epoch_words():
        return [int(torch.as_tensor(tp._DeviceArray(s, (mgb.TP_SYNC_BYTES // 4,)), device="cuda")
                    .view(torch.int32).cpu().numpy()[mgb.TP_EPOCH_OFFSET // 4]) for s in sync]

    graph = None
    try:
        stream = torch.cuda.current_stream()
        x.copy_(torch.from_numpy(synthetic.activations(m, k, seed=50)))
        one_pass(stream.cuda_stream)  # eager: epoch 1
        torch.cuda.synchronize()
        assert epoch_words() == [1, 1]
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(cap):
            with torch.cuda.graph(graph, stream=cap):
                one_pass(torch.cuda.current_stream().cuda_stream)
        stream.wait_stream(cap)
        torch.cuda.synchronize()
        assert epoch_words() == [1, 1]  # capturing runs nothing
        for replay in range(3):
            xh = synthetic.activations(m, k, seed=60 + replay)
            x.copy_(torch.from_numpy(xh))
            for y in ys:
                y.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            assert mgb.take_device_error(torch.cuda.current_device()) == 0
            assert epoch_words() == [2 + replay] * world
            got = [y.cpu().numpy() for y in ys]
            np.testing.assert_array_equal(got[0], got[1])
            np.testing.assert_array_equal(got[0], _plain_shards(torch, fmt, w, n, k, x, world))
    finally:
        del graph
        torch.cuda.synchronize()
        for p in sync:
            mgb.device_free(p)


@pytest.mark.parametrize("fmt_b,n1", [(synthetic.Q4_K, 512), (synthetic.Q8_0, 480)])
@pytest.mark.parametrize("m", [1, 2, 5])
@pytest.mark.parametrize("device_epochs", [False, True])
def test_emulated_two_ranks_chained_call_waits_inside_its_first_kernel(torch_cuda, fmt_b, n1, m,
                                                                        device_epochs):
    """Call B reads call A's gathered y as its x and waits for A's epoch on
    every rank inside its own first kernel (the input wait of mgb_tp_out)
    instead of a wait kernel between the two; only B's own completion is waited
    for.  Ranks emulated one after the other on one GPU; the GEMV (m = 1), the
    tensor-core path (m = 5, the wait in the activation pass) and, for Q8_0 at
    k = 480, the direct-load GEMV in row-pair launches (the first one waits).
    Three rounds; B's gathered y equals the unsharded chain bit for bit."""
    torch = torch_cuda
    world, fmt_a, k, n2 = 2, synthetic.Q4_K, 1024, 256
    wa = synthetic.packed_weights(fmt_a, n1, k, seed=51)
    wb = synthetic.packed_weights(fmt_b, n2, n1, seed=52)
    sa = [_device_layout(torch, fmt_a, tp.shard_packed(fmt_a, wa, n1, k, world, r), n1 // world, k)
          for r in range(world)]
    sb = [_device_layout(torch, fmt_b, tp.shard_packed(fmt_b, wb, n2, n1, world, r), n2 // world, n1)
          for r in range(world)]
    ya = [torch.full((m, n1), float("nan"), dtype=torch.float32, device="cuda") for _ in range(world)]
    yb = [torch.full((m, n2), float("nan"), dtype=torch.float32, device="cuda") for _ in range(world)]
    sync_a = [mgb.device_alloc(mgb.TP_SYNC_BYTES) for _ in range(world)]
    sync_b = [mgb.device_alloc(mgb.TP_SYNC_BYTES) for _ in range(world)]
    ws_bytes = max(mgb.qmatmul_workspace_bytes(fmt_a, m, n1 // world, k),
                   mgb.qmatmul_workspace_bytes(fmt_b, m, n2 // world, n1), 16)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    dev = torch.cuda.current_device()
    try:
        for rnd in range(3):
            e = 0 if device_epochs else rnd + 1
            xd = torch.from_numpy(synthetic.activations(m, k, seed=70 + rnd)).cuda()
            for r in range(world):
                out = mgb.tp_out([y.data_ptr() for y in ya], sync_a, sync_a[r] + mgb.TP_COUNTER_OFFSET,
                                 ldy=n1, col0=r * (n1 // world), epoch=e, rank=r)
                mgb.qmatmul_tp(fmt_a, sa[r].data_ptr(), n1 // world, k, xd.data_ptr(), m, out,
                               workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
            for r in range(world):
                out = mgb.tp_out([y.data_ptr() for y in yb], sync_b, sync_b[r] + mgb.TP_COUNTER_OFFSET,
                                 ldy=n2, col0=r * (n2 // world), epoch=e, rank=r,
                                 wait_done=sync_a[r], wait_epoch=e, wait_world=world)
                mgb.qmatmul_tp(fmt_b, sb[r].data_ptr(), n2 // world, n1, ya[r].data_ptr(), m, out,
                               workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
            for r in range(world):
                mgb.tp_wait(sync_b[r], world, e, 2000, sp)
            torch.cuda.synchronize()
            assert mgb.take_device_error(dev) == 0
            ref_a = _plain_shards(torch, fmt_a, wa, n1, k, xd, world)
            ref_b = _plain_shards(torch, fmt_b, wb, n2, n1, torch.from_numpy(ref_a).cuda(), world)
            for r in range(world):
                np.testing.assert_array_equal(ya[r].cpu().numpy(), ref_a)
                got = yb[r].cpu().numpy()
                bad = np.argwhere(got != ref_b)
                assert bad.size == 0, (rnd, r, sorted(set(bad[:, 0].tolist())),
                                       int(bad[:, 1].min()), int(bad[:, 1].max()), len(bad))
    finally:
        torch.cuda.synchronize()
        for p in sync_a + sync_b:
            mgb.device_free(p)


def test_input_wait_for_an_epoch_nobody_publishes_times_out(torch_cuda):
    """The input wait of a call is bounded like mgb_tp_wait: waiting on an epoch
    no rank publishes gives up, records device error 1, and the context stays
    usable."""
    torch = torch_cuda
    fmt, n, k, m = synthetic.Q4_K, 256, 512, 1
    w = synthetic.packed_weights(fmt, n, k, seed=53)
    wd = _device_layout(torch, fmt, w, n, k)
    xd = torch.from_numpy(synthetic.activations(m, k, seed=54)).cuda()
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    sync, other = mgb.device_alloc(mgb.TP_SYNC_BYTES), mgb.device_alloc(mgb.TP_SYNC_BYTES)
    dev = torch.cuda.current_device()
    try:
        assert mgb.take_device_error(dev) == 0
        out = mgb.tp_out([y.data_ptr()], [sync], sync + mgb.TP_COUNTER_OFFSET, ldy=n, col0=0,
                         epoch=1, rank=0, wait_done=other, wait_epoch=9, wait_world=2,
                         wait_timeout_ms=20)
        mgb.qmatmul_tp(fmt, wd.data_ptr(), n, k, xd.data_ptr(), m, out,
                       stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert mgb.take_device_error(dev) == 1
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
    finally:
        mgb.device_free(sync)
        mgb.device_free(other)


@pytest.mark.parametrize("m", [64, 1])
@pytest.mark.parametrize("epoch", [1, 0])
def test_one_rank_call_publishes_its_completion(torch_cuda, m, epoch):
    """A tensor-parallel call of one rank (split K at m = 64, the sum pass
    before the publish kernel) publishes its epoch, host (1) or device (0), so
    its wait returns at once and y equals the plain call."""
    torch = torch_cuda
    fmt, n, k = synthetic.Q4_K, 512, 1024
    w = synthetic.packed_weights(fmt, n, k, seed=29)
    wd = _device_layout(torch, fmt, w, n, k)
    xd = torch.from_numpy(synthetic.activations(m, k, seed=30)).cuda()
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    sync = mgb.device_alloc(mgb.TP_SYNC_BYTES)
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    try:
        out = mgb.tp_out([y.data_ptr()], [sync], sync + mgb.TP_COUNTER_OFFSET, ldy=n, col0=0,
                         epoch=epoch, rank=0)
        mgb.qmatmul_tp(fmt, wd.data_ptr(), n, k, xd.data_ptr(), m, out,
                       workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=sp)
        mgb.tp_wait(sync, 1, epoch, 2000, sp)
        torch.cuda.synchronize()
        assert mgb.take_device_error(torch.cuda.current_device()) == 0
        got = y.cpu().numpy()
    finally:
        mgb.device_free(sync)
    np.testing.assert_array_equal(got, _plain_shards(torch, fmt, w, n, k, xd))


def test_wait_for_an_epoch_nobody_publishes_times_out(torch_cuda):
    """The bounded wait gives up, records device error 1 and the context stays usable."""
    torch = torch_cuda
    sync = mgb.device_alloc(mgb.TP_SYNC_BYTES)
    try:
        assert mgb.take_device_error(torch.cuda.current_device()) == 0
        mgb.tp_wait(sync, 2, 7, timeout_ms=20, stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert mgb.take_device_error(torch.cuda.current_device()) == 1
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
    finally:
        mgb.device_free(sync)


@pytest.mark.parametrize("device_epochs", [False, True])
def test_reset_after_an_expired_wait(torch_cuda, device_epochs):
    """A wait that gave up leaves the epochs disagreeing; `reset` (every rank
    zeroes its synchronisation words between barriers) makes the next call
    publish and complete again, with the unsharded result."""
    torch = torch_cuda
    fmt, n, k, m = synthetic.Q4_K, 512, 1024, 2
    w = synthetic.packed_weights(fmt, n, k, seed=41)
    xd = torch.from_numpy(synthetic.activations(m, k, seed=42)).cuda()
    op = tp.FusedShardedPackedMatmul(fmt, w, n, k, 1, 0, max_m=m, device_epochs=device_epochs)
    dev = torch.cuda.current_device()
    try:
        ref = _plain_shards(torch, fmt, w, n, k, xd)
        assert np.array_equal(op(xd).cpu().numpy(), ref)
        assert mgb.take_device_error(dev) == 0
        # a peer that never publishes: wait for an epoch nobody reaches
        mgb.tp_wait(op.sync, 1, op.epoch + 5, timeout_ms=20,
                    stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert mgb.take_device_error(dev) == 1
        op.reset()
        words = torch.as_tensor(tp._DeviceArray(op.sync, (mgb.TP_SYNC_BYTES // 4,)),
                                device="cuda").view(torch.int32).cpu().numpy()
        assert not words.any() and op.epoch == 0
        for _ in range(3):
            assert np.array_equal(op(xd).cpu().numpy(), ref)
        assert mgb.take_device_error(dev) == 0
    finally:
        op.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out) -> None:
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    op = None
    try:
        fmt, n, k = synthetic.Q4_K, 1024, 2048
        w = synthetic.packed_weights(fmt, n, k, seed=31)
        op = tp.FusedShardedPackedMatmul(fmt, tp.shard_packed(fmt, w, n, k, world, rank), n, k,
                                         world, rank, max_m=64)
        mismatches = []
        for call, m in enumerate([1, 2, 64, 5, 1, 64]):
            xd = torch.from_numpy(synthetic.activations(m, k, seed=40 + call)).to(dev)
            y = op(xd).cpu().numpy()
            ref = _plain_shards(torch, fmt, w, n, k, xd, world)
            if not np.array_equal(y, ref):
                mismatches.append((call, m, float(np.nanmax(np.abs(y - ref)))))
        # a chained pair: the second call reads the first's gathered y and
        # waits for it inside its own first kernel; one wait at the end
        n2 = 512
        w2 = synthetic.packed_weights(fmt, n2, n, seed=32)
        op2 = tp.FusedShardedPackedMatmul(fmt, tp.shard_packed(fmt, w2, n2, n, world, rank), n2, n,
                                          world, rank, max_m=64)
        try:
            for call, m in enumerate([1, 64, 2]):
                xd = torch.from_numpy(synthetic.activations(m, k, seed=80 + call)).to(dev)
                y1 = op(xd, wait=False)
                y2 = op2(y1, after=op).cpu().numpy()
                ref1 = _plain_shards(torch, fmt, w, n, k, xd, world)
                ref2 = _plain_shards(torch, fmt, w2, n2, n, torch.from_numpy(ref1).to(dev), world)
                if not np.array_equal(y2, ref2):
                    bad = np.argwhere(y2 != ref2)
                    mismatches.append(("chained", call, m, sorted(set(bad[:, 0].tolist()))))
        finally:
            op2.close()
        torch.cuda.synchronize()
        err = mgb.take_device_error(rank)
        out.put((rank, mismatches, err))
    except Exception as e:  # reported to the parent; the barrier below still runs
        out.put((rank, repr(e), -1))
    finally:
        if op is not None:
            op.close()
        dist.destroy_process_group()


def test_two_gpus_fused_gather_matches_plain_shards(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = []
    try:
        for _ in procs:
            results.append(out.get(timeout=300))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for rank, mismatches, err in sorted(results):
        assert mismatches == [] and err == 0, (rank, mismatches, err)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
