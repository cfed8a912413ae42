"""GPU parity at the benchmark configurations' real shapes, through the C ABI.

The reference pins packed matmul against the dense f32 matmul at every shape
it runs (src/native/tests.rs:134-154); here the B200 path is compared with the
C oracle (`ReferenceCpuExecutor` semantics) on the shapes the bench times:

- config 1 (Q4_K, M=512, K=4096, N=14336) on every output column;
- config 3 (Llama-3-8B projections) at M = 1, 16, 64 on every output column,
  with the preferred workspace (split K where the shape takes it) and with the
  minimum one (one K pass);
- config 4 (Llama-3-70B projections) at M = 1 (every column) and M = 2048
  (all rows of sampled columns: 8 M tiles per column tile, K up to 28,672 =
  448 pipeline steps, so the operand rings wrap through many phases);
- `quantize_rows` (src/native/quant.rs:350-378) bit for bit: int8 values, f32
  scales and i32 half sums.

Tolerances as in test_gpu_kernels.py: GEMV (m <= 2) 1e-3, bf16 tensor-core
GEMM 5e-3, normalised by max(1, max|ref|) (src/native/tests.rs:91-103).
The oracle runs over column ranges on a thread pool (ctypes releases the GIL).
"""

from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import magnetar_b200 as mgb
import synthetic
from test_oracle import quantize_edge_rows

pytestmark = pytest.mark.gpu

GEMV_TOL, GEMM_TOL = 1e-3, 5e-3
L8 = [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]  # Wq=Wo, Wk=Wv, gate=up, down
L70 = [(8192, 8192), (1024, 8192), (28672, 8192), (8192, 28672)]


@pytest.fixture(scope="module")
def torch_cuda(cuda_device):
    import torch

    torch.cuda.set_device(cuda_device)
    return torch


def _oracle_columns(oracle, fmt, w, k, x, cols) -> np.ndarray:
    """y[:, cols] from the oracle, column ranges on a thread pool."""
    cols = np.asarray(cols, dtype=np.int64)
    workers = max(1, min(32, os.cpu_count() or 1))
    parts = [p for p in np.array_split(cols, workers * 2) if p.size]

    def one(part):
        return oracle.packed_matmul(fmt, synthetic.row_slice(fmt, w, k, part), len(part), k, x)

    with ThreadPoolExecutor(workers) as pool:
        return np.concatenate(list(pool.map(one, parts)), axis=1)


def _run(torch, fmt, w, n, k, x, min_workspace=False):
    src = torch.from_numpy(w).cuda()
    wdev = torch.empty(mgb.packed_bytes(fmt, n, k), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    mgb.repack(fmt, src.data_ptr(), n, k, wdev.data_ptr(), stream)
    del src
    m = x.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    yd = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    ws_bytes = (mgb.qmatmul_min_workspace_bytes if min_workspace
                else mgb.qmatmul_workspace_bytes)(fmt, m, n, k)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    mgb.qmatmul(fmt, wdev.data_ptr(), n, k, xd.data_ptr(), m, yd.data_ptr(),
                workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=stream)
    torch.cuda.synchronize()
    assert mgb.take_device_error(torch.cuda.current_device()) == 0
    y = yd.cpu().numpy()
    del wdev, xd, yd, ws
    torch.cuda.empty_cache()
    return y


def test_quantize_rows_bit_exact(torch_cuda, oracle):
    torch = torch_cuda
    x = quantize_edge_rows()
    ev, es, esum = oracle.quantize_rows(x)
    xd = torch.from_numpy(x).cuda()
    blocks = x.size // 32
    v = torch.empty(x.size, dtype=torch.int8, device="cuda")
    s = torch.empty(blocks, dtype=torch.float32, device="cuda")
    sm = torch.empty((blocks, 2), dtype=torch.int32, device="cuda")
    mgb.check(mgb.lib().mgb_quantize_rows(xd.data_ptr(), x.size, v.data_ptr(), s.data_ptr(),
                                          sm.data_ptr(), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert np.array_equal(v.cpu().numpy(), ev)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), es.view(np.uint32))
    assert np.array_equal(sm.cpu().numpy(), esum)


def test_config1_every_column(torch_cuda, oracle):
    fmt, m, n, k = mgb.Q4_K, 512, 14336, 4096
    w = synthetic.packed_weights(fmt, n, k)
    x = synthetic.activations(m, k)
    y = _run(torch_cuda, fmt, w, n, k, x)
    ref = _oracle_columns(oracle, fmt, w, k, x, np.arange(n))
    err = oracle.assert_close(y, ref, GEMM_TOL, "config 1, all 14336 columns")
    assert err > 0  # bf16 operands do round


@pytest.mark.parametrize("n,k", L8)
@pytest.mark.parametrize("m", [1, 16, 64])
def test_config3_projection(torch_cuda, oracle, m, n, k):
    fmt = mgb.Q4_K
    w = synthetic.packed_weights(fmt, n, k, seed=n + k)
    x = synthetic.activations(m, k, seed=k)
    ref = _oracle_columns(oracle, fmt, w, k, x, np.arange(n))
    tol = GEMV_TOL if m <= 2 else GEMM_TOL
    y = _run(torch_cuda, fmt, w, n, k, x)
    oracle.assert_close(y, ref, tol, f"config 3 m {m} n {n} k {k}")
    if m > 2:  # one K pass as well (the tensor-parallel calls run this form)
        y1 = _run(torch_cuda, fmt, w, n, k, x, min_workspace=True)
        oracle.assert_close(y1, ref, tol, f"config 3 one pass m {m} n {n} k {k}")


@pytest.mark.parametrize("n,k", L70)
def test_config4_decode_every_column(torch_cuda, oracle, n, k):
    fmt = mgb.Q4_K
    w = synthetic.packed_weights(fmt, n, k, seed=n + k)
    x = synthetic.activations(1, k, seed=k)
    y = _run(torch_cuda, fmt, w, n, k, x)
    oracle.assert_close(y, _oracle_columns(oracle, fmt, w, k, x, np.arange(n)), GEMV_TOL,
                        f"config 4 m 1 n {n} k {k}")


@pytest.mark.parametrize("n,k", L70)
def test_config4_prefill_sampled_columns(torch_cuda, oracle, n, k):
    """M = 2048: every row of 96 columns spread over all column tiles plus the
    last 16 columns."""
    fmt, m = mgb.Q4_K, 2048
    w = synthetic.packed_weights(fmt, n, k, seed=n + k)
    x = synthetic.activations(m, k, seed=k)
    y = _run(torch_cuda, fmt, w, n, k, x)
    assert np.isfinite(y).all()
    cols = np.unique(np.concatenate([np.linspace(0, n - 1, 96).astype(np.int64),
                                     np.arange(n - 16, n)]))
    ref = _oracle_columns(oracle, fmt, w, k, x, cols)
    err = oracle.assert_close(y[:, cols], ref, GEMM_TOL, f"config 4 m {m} n {n} k {k}")
    assert err > 0
