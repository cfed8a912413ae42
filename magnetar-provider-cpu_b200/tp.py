"""Tensor parallelism of the packed matmul over output columns.

A packed weight's stored rows are the matmul's output columns, and each stored
row is a whole sequence of blocks, so the rows split across ranks without
touching a block: rank g of G holds stored rows [g N/G, (g+1) N/G) (the unit the
reference's CPU pool partitions on, `packed_matmul`, src/native/mod.rs:135-150).
Every rank multiplies the same activations by its shard and every rank ends
with the full [M, N].  Two exchanges:

- `FusedShardedPackedMatmul` (the B200 path): the kernels store each output
  column straight into every rank's y over NVLink (peers' buffers mapped with
  CUDA IPC), then publish the call's epoch; a rank waits for all epochs with
  one stream-ordered kernel (`mgb_qmatmul_tp`, `mgb_tp_wait`).  No collective
  launch, no gather buffer, no interleave pass: the transfer overlaps the tiles
  still computing.
- `ShardedPackedMatmul` + `gather_columns`: the rank's [M, N/G] block, then an
  NCCL (gloo on CPU, for the host logic's tests) all-gather and an interleave
  back to [M, N] — the library baseline.
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


class _DeviceArray:
    """A raw device pointer as a CUDA array (for torch.as_tensor)."""

    def __init__(self, ptr: int, shape: tuple[int, ...]):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class FusedShardedPackedMatmul(ShardedPackedMatmul):
    """The sharded matmul with the all-gather fused into the kernels' stores.

    Each rank owns two y buffers of [max_m, N] f32 and 256 bytes of
    synchronisation words (`mgb_device_alloc`), and maps every peer's with CUDA
    IPC (handles exchanged once with `all_gather_object`).  Call e writes into
    buffer e % 2 of every rank, then waits (on the stream) until every rank has
    published epoch e.  The returned tensor views this rank's buffer: it stays
    valid until the call after next, which rewrites it.  Two buffers suffice:
    rank A writes buffer b for call e+2 only after it has seen every peer's
    epoch e+1, and a peer publishes e+1 only after its stream has finished all
    work queued before that call, including its reads of call e's result."""

    def __init__(self, fmt: int, ggml_shard: np.ndarray, n: int, k: int, world: int, rank: int,
                 max_m: int, group=None, device=None, timeout_ms: int = 2000,
                 device_epochs: bool = False):
        import torch.distributed as dist

        import magnetar_b200 as mgb

        super().__init__(fmt, ggml_shard, n, k, world, rank, device)
        if world > mgb.MAX_TP:
            raise ValueError(f"at most {mgb.MAX_TP} ranks")
        self.max_m, self.group, self.timeout_ms = max_m, group, timeout_ms
        # device epochs: the kernels and the wait take the epoch from this
        # rank's epoch word, so calls captured in a CUDA graph (an even number
        # of them, for the buffer alternation) replay with fresh epochs
        self.device_epochs = device_epochs
        self._own: list[int] = []
        self._mapped: list[int] = []
        try:
            self.sync = self._alloc(mgb.TP_SYNC_BYTES)
            self.slots = [self._alloc(max_m * n * 4) for _ in range(2)]
            mine = [mgb.ipc_handle(p) for p in (self.sync, *self.slots)]
            handles: list = [None] * world
            if world > 1:
                dist.all_gather_object(handles, mine, group=group)
            else:
                handles = [mine]
            peers = []
            for r, hs in enumerate(handles):
                if r == rank:
                    peers.append((self.sync, *self.slots))
                else:
                    ptrs = []
                    for h in hs:
                        ptrs.append(mgb.ipc_open(h))
                        self._mapped.append(ptrs[-1])
                    peers.append(tuple(ptrs))
            if world > 1:
                dist.barrier(group=group)
        except Exception:
            self.close()
            raise
        self.done = [p[0] for p in peers]
        self.y_slots = [[p[1 + s] for p in peers] for s in range(2)]
        self.epoch = 0

    def _alloc(self, nbytes: int) -> int:
        import magnetar_b200 as mgb

        ptr = mgb.device_alloc(nbytes)
        self._own.append(ptr)
        return ptr

    def __call__(self, x, group=None, after=None, wait=True):
        """y [M, N] (every rank's columns) for device activations x [M, K] (f32).

        `after`: the fused op whose latest call on this stream produced x (or
        must otherwise complete first); this call's first kernel waits for that
        call's epoch on every rank before reading x, instead of a wait kernel
        of its own between the two.  `wait=False` leaves this call's own wait
        to whoever consumes y: a later call with after=self, or wait()."""
        import torch

        import magnetar_b200 as mgb

        m = x.shape[0]
        if not 0 < m <= self.max_m:
            raise ValueError(f"{m} activation rows (1..{self.max_m})")
        if after is not None and after.device_epochs != self.device_epochs:
            raise ValueError("chained fused calls use one epoch mode")
        self.epoch += 1
        slot = self.epoch & 1
        epoch = 0 if self.device_epochs else self.epoch
        wait_kw = {}
        if after is not None:
            wait_kw = dict(wait_done=after.sync, wait_world=after.world,
                           wait_epoch=0 if after.device_epochs else after.epoch,
                           wait_timeout_ms=after.timeout_ms)
        out = mgb.tp_out(self.y_slots[slot], self.done, self.sync + mgb.TP_COUNTER_OFFSET,
                         ldy=self.n, col0=self.rank * self.n_loc, epoch=epoch, rank=self.rank,
                         **wait_kw)
        ws_bytes = mgb.qmatmul_workspace_bytes(self.fmt, m, self.n_loc, self.k)
        if ws_bytes and (self._ws is None or self._ws.numel() < ws_bytes):
            self._ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.device)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        mgb.qmatmul_tp(self.fmt, self.weight.data_ptr(), self.n_loc, self.k, x.data_ptr(), m, out,
                       workspace_ptr=self._ws.data_ptr() if ws_bytes else 0,
                       workspace_bytes=ws_bytes, stream=stream)
        if wait:
            self.wait()
        return torch.as_tensor(_DeviceArray(self.slots[slot], (m, self.n)), device=self.device)

    def wait(self) -> None:
        """Stream-ordered wait for this op's latest call on every rank."""
        import torch

        import magnetar_b200 as mgb

        mgb.tp_wait(self.sync, self.world, 0 if self.device_epochs else self.epoch,
                    self.timeout_ms, torch.cuda.current_stream(self.device).cuda_stream)

    def reset(self) -> None:
        """Recovery after a wait gave up (device error 1, a peer that never
        published): the ranks' epochs then disagree and every later wait would
        expire too.  Collective: every rank drains its stream, all ranks zero
        their synchronisation words (reserved word, epoch word, done words) between
        two barriers, and epochs restart from 1."""
        import torch
        import torch.distributed as dist

        import magnetar_b200 as mgb

        multi = self.world > 1 and dist.is_initialized()
        torch.cuda.synchronize(self.device)
        if multi:
            dist.barrier(group=self.group)
        torch.as_tensor(_DeviceArray(self.sync, (mgb.TP_SYNC_BYTES // 4,)),
                        device=self.device).zero_()
        torch.cuda.synchronize(self.device)
        if multi:
            dist.barrier(group=self.group)
        self.epoch = 0

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's.  Collective: every
        rank calls it (no peer may still be writing into this rank's buffers)."""
        import torch
        import torch.distributed as dist

        import magnetar_b200 as mgb

        torch.cuda.synchronize(self.device)
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)
        for p in self._mapped:
            mgb.ipc_close(p)
        for p in self._own:
            mgb.device_free(p)
        self._mapped, self._own = [], []
