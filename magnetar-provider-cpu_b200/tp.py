"""Tensor parallelism of the packed matmul over output columns.

A packed weight's stored rows are the matmul's output columns, and each stored
row is a whole sequence of blocks, so the rows split across ranks without
touching a block: rank g of G holds stored rows [g N/G, (g+1) N/G) (the unit the
reference's CPU pool partitions on, `packed_matmul`, src/native/mod.rs:135-150).
Every rank multiplies the same activations by its shard; the [M, N/G] outputs
are then all-gathered (NCCL over NVLink between B200s; gloo on CPU for the host
logic's tests) and interleaved back to [M, N].

This module is the host side of the multi-GPU path: it owns the sharding and the
exchange, the kernels stay the single-GPU ones.
"""

from __future__ import annotations

import numpy as np

import synthetic


def shard_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """Stored rows [lo, hi) of `rank` for an N-row weight over `world` ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n % world:
        raise ValueError(f"{n} output columns do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_packed(fmt: int, ggml: np.ndarray, n: int, k: int, world: int, rank: int) -> np.ndarray:
    """The checkpoint bytes (ggml blocks) of this rank's stored rows: one
    contiguous byte range, stored_row_bytes * N/G long."""
    lo, hi = shard_bounds(n, world, rank)
    row_bytes = synthetic.packed_nbytes(fmt, 1, k)
    flat = np.ascontiguousarray(ggml, dtype=np.uint8).reshape(-1)
    if flat.size != n * row_bytes:
        raise ValueError(f"{flat.size} bytes are not {n} rows of {row_bytes}")
    return flat[lo * row_bytes:hi * row_bytes]


def gather_columns(y_local, group=None):
    """All-gathers each rank's [M, N/G] output and returns the full [M, N]
    (rank g's columns at [g N/G, (g+1) N/G)).  `y_local` is a torch tensor on
    the backend's device (CUDA for NCCL, CPU for gloo)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    m, n_loc = y_local.shape
    y_local = y_local.contiguous()
    if world == 1:
        return y_local
    parts = torch.empty((world, m, n_loc), dtype=y_local.dtype, device=y_local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(parts.view(-1), y_local.view(-1), group=group)
    else:
        dist.all_gather(list(parts.unbind(0)), y_local, group=group)
    return parts.permute(1, 0, 2).reshape(m, world * n_loc)


class ShardedPackedMatmul:
    """One rank's shard of a packed weight, resident on this rank's GPU in the
    device layout, and the sharded matmul y = x W^T with the output all-gathered.

    The weight bytes are this rank's shard (`shard_packed`); the local product
    runs `mgb_qmatmul` on the current CUDA stream."""

    def __init__(self, fmt: int, ggml_shard: np.ndarray, n: int, k: int, world: int, rank: int,
                 device=None):
        import torch

        import magnetar_b200 as mgb

        self.fmt, self.n, self.k, self.world, self.rank = fmt, n, k, world, rank
        self.n_loc = n // world
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        stream = torch.cuda.current_stream(self.device).cuda_stream
        src = torch.from_numpy(np.ascontiguousarray(ggml_shard)).to(self.device)
        self.weight = torch.empty(mgb.packed_bytes(fmt, self.n_loc, k), dtype=torch.uint8,
                                  device=self.device)
        mgb.repack(fmt, src.data_ptr(), self.n_loc, k, self.weight.data_ptr(), stream)
        self._ws = None

    def local(self, x, out=None):
        """This rank's [M, N/G] columns for device activations x [M, K] (f32)."""
        import torch

        import magnetar_b200 as mgb

        m = x.shape[0]
        y = out if out is not None else torch.empty((m, self.n_loc), dtype=torch.float32,
                                                    device=self.device)
        ws_bytes = mgb.qmatmul_workspace_bytes(self.fmt, m, self.n_loc, self.k)
        if ws_bytes and (self._ws is None or self._ws.numel() < ws_bytes):
            self._ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.device)
        mgb.qmatmul(self.fmt, self.weight.data_ptr(), self.n_loc, self.k, x.data_ptr(), m,
                    y.data_ptr(), workspace_ptr=self._ws.data_ptr() if ws_bytes else 0,
                    workspace_bytes=ws_bytes,
                    stream=torch.cuda.current_stream(self.device).cuda_stream)
        return y

    def __call__(self, x, group=None):
        return gather_columns(self.local(x), group)
