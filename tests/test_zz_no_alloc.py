"""mgb_qmatmul_static_scratch: the packed-weight matmul for callers that must
not allocate device memory (a runtime that reserves the GPU for its own arena,
or a hot path that must stay out of the driver's allocator).

Its output must equal the allocating entry point's (mgb_qmatmul with a
caller-provided workspace) within the tolerance the parity tests use, on two
calls in a row: the second call runs on the shared static array still holding
the first call's bytes.  The file is named to be collected last, and it passes
both alone in a fresh process and after the other GPU tests.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import magnetar_b200 as mgb
import synthetic

pytestmark = pytest.mark.gpu
GEMV_TOL, GEMM_TOL = 1e-3, 5e-3


def _norm_err(a: np.ndarray, b: np.ndarray) -> float:
    scale = max(1.0, float(np.max(np.abs(b))))
    return float(np.max(np.abs(a.astype(np.float64) - b.astype(np.float64)))) / scale


@pytest.mark.parametrize(
    "fmt,m,n,k",
    [(mgb.Q4_K, 512, 14336, 4096),   # tensor-core path, 4 MiB of the 8 MiB scratch
     (mgb.Q4_K, 64, 300, 512),
     (mgb.IQ4_NL, 9, 37, 512),
     (mgb.Q8_0, 1, 4096, 4096)])     # GEMV path: no scratch touched
def test_static_scratch_matches_allocating_entry(cuda_device, fmt, m, n, k):
    import torch

    torch.cuda.set_device(cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    w = synthetic.packed_weights(fmt, n, k, seed=17)
    src = torch.from_numpy(w).cuda()
    wdev = torch.empty(mgb.packed_bytes(fmt, n, k), dtype=torch.uint8, device="cuda")
    mgb.repack(fmt, src.data_ptr(), n, k, wdev.data_ptr(), stream)
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n, k)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device="cuda")
    tol = GEMV_TOL if m <= 2 else GEMM_TOL
    for call in range(2):  # two calls in a row, different activations
        x = torch.from_numpy(synthetic.activations(m, k, seed=100 + call)).cuda()
        y_ref = torch.full((m, n), float("nan"), device="cuda")
        y = torch.full((m, n), float("nan"), device="cuda")
        mgb.qmatmul(fmt, wdev.data_ptr(), n, k, x.data_ptr(), m, y_ref.data_ptr(),
                    workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=stream)
        mgb.check(mgb.lib().mgb_qmatmul_static_scratch(fmt, wdev.data_ptr(), n, k, x.data_ptr(),
                                                       m, y.data_ptr(), None, 0, stream))
        torch.cuda.synchronize()
        a, b = y.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(a).all(), f"call {call}: non-finite output"
        assert _norm_err(a, b) <= tol, f"call {call}: {_norm_err(a, b)} > {tol}"


def test_static_scratch_back_to_back_calls_allocate_nothing(cuda_device):
    """Two calls queued on one stream with nothing between them (split K active:
    the shared array holds the bf16 activations and the partial planes), with
    different activations: each output equals the allocating entry point's, and
    neither torch's allocator nor the device's free memory moves."""
    import torch

    torch.cuda.set_device(cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    fmt, m, n, k = mgb.Q4_K, 16, 4096, 4096
    assert mgb.qmatmul_workspace_bytes(fmt, m, n, k) > mgb.qmatmul_min_workspace_bytes(fmt, m, n, k)
    w = synthetic.packed_weights(fmt, n, k, seed=19)
    src = torch.from_numpy(w).cuda()
    wdev = torch.empty(mgb.packed_bytes(fmt, n, k), dtype=torch.uint8, device="cuda")
    mgb.repack(fmt, src.data_ptr(), n, k, wdev.data_ptr(), stream)
    ws_bytes = mgb.qmatmul_workspace_bytes(fmt, m, n, k)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    xs = [torch.from_numpy(synthetic.activations(m, k, seed=200 + i)).cuda() for i in range(2)]
    refs = [torch.full((m, n), float("nan"), device="cuda") for _ in range(2)]
    ys = [torch.full((m, n), float("nan"), device="cuda") for _ in range(2)]
    for x, r in zip(xs, refs):
        mgb.qmatmul(fmt, wdev.data_ptr(), n, k, x.data_ptr(), m, r.data_ptr(),
                    workspace_ptr=ws.data_ptr(), workspace_bytes=ws_bytes, stream=stream)
    # one call first, so that lazy module loading is not counted below
    mgb.check(mgb.lib().mgb_qmatmul_static_scratch(fmt, wdev.data_ptr(), n, k, xs[0].data_ptr(),
                                                   m, ys[0].data_ptr(), None, 0, stream))
    torch.cuda.synchronize()
    allocated, free = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]
    for x, y in zip(xs, ys):
        mgb.check(mgb.lib().mgb_qmatmul_static_scratch(fmt, wdev.data_ptr(), n, k, x.data_ptr(),
                                                       m, y.data_ptr(), None, 0, stream))
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == allocated
    assert torch.cuda.mem_get_info()[0] == free
    assert mgb.take_device_error(cuda_device) == 0
    for call, (y, r) in enumerate(zip(ys, refs)):
        a, b = y.cpu().numpy(), r.cpu().numpy()
        assert np.isfinite(a).all(), f"call {call}: non-finite output"
        assert _norm_err(a, b) <= GEMM_TOL, f"call {call}: {_norm_err(a, b)} > {GEMM_TOL}"
    assert not np.array_equal(ys[0].cpu().numpy(), ys[1].cpu().numpy())


def test_static_scratch_rejects_oversized_shapes(cuda_device):
    import torch

    torch.cuda.set_device(cuda_device)
    limit = mgb.lib().mgb_qmatmul_static_scratch
    # m * k = 1024 * 8192 needs 16 MiB of bf16 scratch: refused before any device work
    dummy = ctypes.c_void_p(16)
    status = limit(mgb.Q4_K, dummy, 256, 8192, dummy, 1024, dummy, None, 0, None)
    assert status == mgb.INVALID_ARGUMENT
    assert "static scratch holds 8388608" in mgb.last_error()
