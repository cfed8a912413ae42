"""Tensor-parallel host logic on CPU (no GPU): sharding by stored rows and the
all-gather of output columns.

Two `gloo` ranks shard a packed weight by stored rows, compute their column
blocks with the CPU oracle, all-gather and interleave them.  The result must equal
the unsharded product bit for bit, since every output column is computed
independently (`packed_matmul`, src/native/mod.rs:135-150, partitions the same
way across its thread pool).
"""

from __future__ import annotations

import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import synthetic
import tp


def test_shard_bounds_cover_every_row_once():
    n, world = 14336, 8
    spans = [tp.shard_bounds(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        tp.shard_bounds(100, 3, 0)
    with pytest.raises(ValueError):
        tp.shard_bounds(64, 2, 2)


@pytest.mark.parametrize("fmt", [synthetic.Q4_K, synthetic.Q8_0, synthetic.IQ4_NL])
def test_shards_are_the_stored_rows(oracle, fmt):
    n, k, world = 64, 512, 4
    w = synthetic.packed_weights(fmt, n, k, seed=3)
    full = oracle.dequantize(fmt, w, n, k).reshape(n, k)
    for rank in range(world):
        lo, hi = tp.shard_bounds(n, world, rank)
        shard = tp.shard_packed(fmt, w, n, k, world, rank)
        assert shard.size == synthetic.packed_nbytes(fmt, hi - lo, k)
        np.testing.assert_array_equal(oracle.dequantize(fmt, shard, hi - lo, k).reshape(hi - lo, k),
                                      full[lo:hi])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, fmt: int, n: int, k: int, m: int, out) -> None:
    import torch
    import torch.distributed as dist

    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        w = synthetic.packed_weights(fmt, n, k, seed=11)
        x = synthetic.activations(m, k, seed=12)
        shard = tp.shard_packed(fmt, w, n, k, world, rank)
        y_loc = oracle.packed_matmul(fmt, shard, n // world, k, x)
        y = tp.gather_columns(torch.from_numpy(y_loc))
        if rank == 0:
            out.put(y.numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,n,k,m", [(synthetic.Q4_K, 512, 512, 3),
                                       (synthetic.Q8_0, 256, 128, 1),
                                       (synthetic.IQ4_NL, 64, 96, 2)])
def test_two_gloo_ranks_match_the_unsharded_product(oracle, fmt, n, k, m):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, fmt, n, k, m, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        y = out.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    w = synthetic.packed_weights(fmt, n, k, seed=11)
    x = synthetic.activations(m, k, seed=12)
    np.testing.assert_array_equal(y, oracle.packed_matmul(fmt, w, n, k, x))
