"""GPU parity of the B200 kernels against the CPU oracle, through the C ABI.

Tolerances, normalised as the reference does
(src/native/tests.rs:91-103: |a - e| <= tol * max(1, max|e|)):
  dequantisation          bit-exact
  GEMV (f32, m <= 2)      1e-3
  tensor-core GEMM (bf16) 5e-3
"""

from __future__ import annotations

import pathlib

import numpy as np
import pytest

import magnetar_b200 as mgb
import synthetic

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "dequant_gguf.npz"
FORMATS = [mgb.Q4_K, mgb.Q5_K, mgb.Q6_K, mgb.Q8_0, mgb.IQ4_NL, mgb.Q4_0]
GEMV_TOL, GEMM_TOL = 1e-3, 5e-3


@pytest.fixture(scope="module")
def torch_cuda(cuda_device):
    import torch

    torch.cuda.set_device(cuda_device)
    return torch


def _device_layout(torch, fmt, ggml: np.ndarray, rows: int, cols: int):
    src = torch.from_numpy(np.ascontiguousarray(ggml)).cuda()
    out = torch.empty(mgb.packed_bytes(fmt, rows, cols), dtype=torch.uint8, device="cuda")
    mgb.repack(fmt, src.data_ptr(), rows, cols, out.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out


def _qmatmul(torch, fmt, wdev, n, k, x: np.ndarray, addend: np.ndarray | None = None,
             min_workspace: bool = False):
    m = x.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    yd = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    ws_bytes = (mgb.qmatmul_min_workspace_bytes if min_workspace
                else mgb.qmatmul_workspace_bytes)(fmt, m, n, k)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    ad = None
    if addend is not None:
        ad = torch.from_numpy(np.ascontiguousarray(addend, dtype=np.float32)).cuda()
    mgb.qmatmul(fmt, wdev.data_ptr(), n, k, xd.data_ptr(), m, yd.data_ptr(),
                ad.data_ptr() if ad is not None else 0, ad.numel() if ad is not None else 0,
                ws.data_ptr(), ws_bytes, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert mgb.take_device_error(torch.cuda.current_device()) == 0
    return yd.cpu().numpy()


def _same_bits(a, b):
    nan = np.isnan(a)
    assert np.array_equal(nan, np.isnan(b))
    return np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("name", ["q4_k", "q5_k", "q6_k", "q8_0", "iq4_nl", "q4_0"])
@pytest.mark.parametrize("source", ["reference_generator", "random_bytes"])
def test_dequantize_bit_exact_to_gguf_and_oracle(torch_cuda, oracle, name, source):
    torch = torch_cuda
    golden = np.load(GOLDEN)
    key = f"{name}__{source}"
    fmt, rows, cols = (int(v) for v in golden[key + "__meta"])
    data = golden[key + "__bytes"]
    wdev = _device_layout(torch, fmt, data, rows, cols)
    out = torch.empty((rows, cols), dtype=torch.float32, device="cuda")
    mgb.dequantize(fmt, wdev.data_ptr(), rows, cols, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert _same_bits(got, golden[key + "__expected"])
    assert _same_bits(got, oracle.dequantize(fmt, data, rows, cols))


@pytest.mark.parametrize("fmt", FORMATS)
def test_dequantize_full_size_bit_exact(torch_cuda, oracle, fmt):
    torch = torch_cuda
    n, k = 4096, 4096
    w = synthetic.packed_weights(fmt, n, k, seed=3)
    wdev = _device_layout(torch, fmt, w, n, k)
    out = torch.empty((n, k), dtype=torch.float32, device="cuda")
    mgb.dequantize(fmt, wdev.data_ptr(), n, k, out.data_ptr())
    torch.cuda.synchronize()
    assert _same_bits(out.cpu().numpy(), oracle.dequantize(fmt, w, n, k))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 2])
@pytest.mark.parametrize("n,k", [(37, 512), (5, 96), (300, 8192), (64, 14336), (16, 32768),
                                 (24, 40960), (9, 32800)])
def test_gemv_parity(torch_cuda, oracle, fmt, m, n, k):
    """Down to K = 96 and up past 1,024 runs (K = 40,960 and the ragged 32,800:
    more runs than a CTA has threads, each thread taking several)."""
    if fmt in (mgb.Q4_K, mgb.Q5_K, mgb.Q6_K) and k % 256:
        pytest.skip("the K-quant formats need whole 256-value super-blocks")
    torch = torch_cuda
    w = oracle.test_packed(fmt, n, k, 21)  # the reference's own test generator
    x = oracle.test_activations(m, k, m)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    ref = oracle.packed_matmul(fmt, w, n, k, x)
    err = oracle.assert_close(y, ref, GEMV_TOL, f"gemv fmt {fmt} m {m} n {n} k {k}")
    # activations held as 16-bit integers per 32-value run (|error| <= 2^-16 of
    # the run's largest value), exact integer dots: ~2e-5, far inside 1e-3
    assert err < 1e-4


@pytest.mark.parametrize("fmt", [mgb.Q8_0, mgb.IQ4_NL])
def test_ragged_large_k_batch(torch_cuda, oracle, fmt):
    """m = 3 with K = 32,800 (a multiple of 32, not of 256): no tensor-core form
    applies, so the rows go in pairs through the direct-load GEMV, whose
    threads each take two runs."""
    torch = torch_cuda
    m, n, k = 3, 40, 32800
    w = oracle.test_packed(fmt, n, k, 23)
    x = oracle.test_activations(m, k, 5)
    y = _qmatmul(torch, fmt, _device_layout(torch, fmt, w, n, k), n, k, x)
    oracle.assert_close(y, oracle.packed_matmul(fmt, w, n, k, x), GEMV_TOL, f"fmt {fmt} k {k}")


@pytest.mark.parametrize("fmt", [mgb.Q4_K])
def test_gemv_config0_q4k_4096(torch_cuda, oracle, fmt):
    torch = torch_cuda
    n = k = 4096
    w = synthetic.packed_weights(fmt, n, k)
    x = synthetic.activations(1, k)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    y2 = _qmatmul(torch, fmt, wdev, n, k, x)
    assert np.array_equal(y, y2), "GEMV is deterministic"
    oracle.assert_close(y, oracle.packed_matmul(fmt, w, n, k, x), GEMV_TOL, "config 0")


@pytest.mark.parametrize("fmt", [mgb.Q8_0, mgb.IQ4_NL, mgb.Q6_K, mgb.Q5_K])
@pytest.mark.parametrize("m", [1, 8])
def test_config2_mixed_formats(torch_cuda, oracle, fmt, m):
    torch = torch_cuda
    n, k = 14336, 4096
    w = synthetic.packed_weights(fmt, n, k)
    x = synthetic.activations(m, k)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    tol = GEMV_TOL if m <= 2 else GEMM_TOL
    oracle.assert_close(y, oracle.packed_matmul(fmt, w, n, k, x), tol, f"config 2 fmt {fmt} m {m}")


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [3, 9, 64, 130, 300])
def test_gemm_parity(torch_cuda, oracle, fmt, m):
    torch = torch_cuda
    n, k = 300, 512
    w = oracle.test_packed(fmt, n, k, 31)
    x = oracle.test_activations(m, k, m)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    oracle.assert_close(y, oracle.packed_matmul(fmt, w, n, k, x), GEMM_TOL, f"gemm fmt {fmt} m {m}")


def test_gemm_config1_sampled_columns(torch_cuda, oracle):
    """Config 1 (X[512,4096] x Q4_K W[14336 x 4096]) at full size on the GPU;
    the oracle checks 320 output columns spread over every column tile,
    including the last, against all 512 rows."""
    torch = torch_cuda
    fmt, m, n, k = mgb.Q4_K, 512, 14336, 4096
    w = synthetic.packed_weights(fmt, n, k)
    x = synthetic.activations(m, k)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    assert np.isfinite(y).all()
    cols = np.unique(np.concatenate([np.linspace(0, n - 1, 300).astype(np.int64),
                                     np.arange(n - 20, n)]))
    sub = synthetic.row_slice(fmt, w, k, cols)
    ref = oracle.packed_matmul(fmt, sub, len(cols), k, x)
    err = oracle.assert_close(y[:, cols], ref, GEMM_TOL, "config 1")
    assert err > 0  # bf16 operands do round
    y2 = _qmatmul(torch, fmt, wdev, n, k, x)
    assert np.array_equal(y, y2), "GEMM is deterministic (no split-K atomics)"


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m,n,k,parts", [(3, 300, 1024, 4), (64, 8192, 4096, 2),
                                         (128, 1001, 2048, 8), (17, 64, 14336, 8),
                                         (8, 512, 1536, 2), (64, 14336, 4096, 1),
                                         (16, 4096, 4096, 4), (200, 1000, 1024, 4),
                                         (512, 1792, 4096, 4), (256, 1792, 4096, 8),
                                         (512, 1024, 8192, 8), (512, 3584, 8192, 2),
                                         (512, 3584, 4096, 1), (600, 1024, 8192, 4),
                                         (2048, 128, 8192, 8), (2048, 512, 8192, 4),
                                         (2048, 1024, 28672, 2),
                                         (1024, 256, 8192, 8)])
def test_gemm_split_k(torch_cuda, oracle, fmt, m, n, k, parts):
    """With the preferred workspace a call with narrow tiles (or, for 129..512
    rows, a long K) splits K over 2, 4 or 8 CTAs per tile and
    sums the parts in a fixed order: the result is deterministic and matches
    the one-pass call (minimum workspace) to within the GEMM tolerance."""
    torch = torch_cuda
    planes = 0 if parts == 1 else parts
    assert mgb.qmatmul_workspace_bytes(fmt, m, n, k) == \
        mgb.qmatmul_min_workspace_bytes(fmt, m, n, k) + planes * m * n * 4
    w = synthetic.packed_weights(fmt, n, k, seed=m + k)
    x = synthetic.activations(m, k, seed=n)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    assert np.isfinite(y).all()
    assert np.array_equal(y, _qmatmul(torch, fmt, wdev, n, k, x)), "deterministic"
    one = _qmatmul(torch, fmt, wdev, n, k, x, min_workspace=True)
    oracle.assert_close(y, one, GEMM_TOL, f"split vs one pass fmt {fmt} m {m} n {n}")
    cols = np.unique(np.concatenate([np.linspace(0, n - 1, 64).astype(np.int64),
                                     np.arange(max(0, n - 8), n)]))
    ref = oracle.packed_matmul(fmt, synthetic.row_slice(fmt, w, k, cols), len(cols), k, x)
    oracle.assert_close(y[:, cols], ref, GEMM_TOL, f"split K fmt {fmt} m {m} n {n} k {k}")
    # the sum pass adds a bias row or a residual after the halves
    bias = np.linspace(-2, 2, n, dtype=np.float32)
    yb = _qmatmul(torch, fmt, wdev, n, k, x, bias)
    assert np.array_equal(yb, (y + bias).astype(np.float32))
    res = synthetic.activations(m, n, seed=k)
    yr = _qmatmul(torch, fmt, wdev, n, k, x, res)
    assert np.array_equal(yr, (y + res).astype(np.float32))


@pytest.mark.parametrize("m", [1, 2, 64, 300])
def test_addend_epilogues(torch_cuda, oracle, m):
    torch = torch_cuda
    fmt, n, k = mgb.Q4_K, 96, 512
    w = oracle.test_packed(fmt, n, k, 5)
    x = oracle.test_activations(m, k, 9)
    wdev = _device_layout(torch, fmt, w, n, k)
    tol = GEMV_TOL if m <= 2 else GEMM_TOL
    base = oracle.packed_matmul(fmt, w, n, k, x)
    bias = np.linspace(-3, 3, n, dtype=np.float32)
    oracle.assert_close(_qmatmul(torch, fmt, wdev, n, k, x, bias), oracle.add(base, bias), tol)
    resid = oracle.test_activations(m, n, 11)
    oracle.assert_close(_qmatmul(torch, fmt, wdev, n, k, x, resid), oracle.add(resid, base), tol)
    # fused equals unfused bit for bit, as the reference requires of matmul-bias /
    # matmul-residual against matmul then add (src/tests.rs:740-888)
    plain = _qmatmul(torch, fmt, wdev, n, k, x)
    assert np.array_equal(_qmatmul(torch, fmt, wdev, n, k, x, bias), plain + bias[None, :])
    assert np.array_equal(_qmatmul(torch, fmt, wdev, n, k, x, resid), resid + plain)


@pytest.mark.parametrize("fmt", FORMATS)
def test_input_major_parity(torch_cuda, oracle, fmt):
    torch = torch_cuda
    rows, cols = 64, 256  # stored rows = input rows
    w = oracle.test_packed(fmt, rows, cols, 61)
    wdev = _device_layout(torch, fmt, w, rows, cols)
    for m in (1, 4):
        x = oracle.test_activations(m, rows, 62)
        x[0, 3] = 0.0  # the reference skips zero activations
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((m, cols), dtype=torch.float32, device="cuda")
        mgb.qmatmul_input_major(fmt, wdev.data_ptr(), rows, cols, xd.data_ptr(), m, yd.data_ptr())
        torch.cuda.synchronize()
        ref = oracle.packed_axpy(fmt, w, rows, cols, x)
        assert np.array_equal(yd.cpu().numpy(), ref)  # same order, same roundings


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("m", [1, 2, 5])
def test_nan_activation_reaches_its_row_only(torch_cuda, oracle, fmt, m):
    """A NaN activation makes its whole output row NaN and leaves the other rows
    finite, as the reference's f32 matmul does (x * w is NaN for every w)."""
    n, k = 96, 512
    w = synthetic.packed_weights(fmt, n, k, seed=21)
    wdev = _device_layout(torch_cuda, fmt, w, n, k)
    x = synthetic.activations(m, k, seed=22)
    x[0, 37] = np.nan
    y = _qmatmul(torch_cuda, fmt, wdev, n, k, x)
    ref = oracle.packed_matmul(fmt, w, n, k, x)
    assert np.isnan(ref[0]).all()
    assert np.isnan(y[0]).all(), f"{np.isnan(y[0]).sum()} of {n} NaN in row 0"
    assert np.isfinite(y[1:]).all()


@pytest.mark.parametrize("m,n,k", [(40, 28672, 256), (300, 14344, 256), (300, 14342, 256),
                                   (16, 65536, 256)])
def test_gemm_wide_tile_epilogue_edges(torch_cuda, oracle, m, n, k):
    """Wide tiles (bn >= 192) store 32x32 output blocks by TMA: rows past m and
    columns past n are clipped by the tensor map, a tile's partial last block
    (bn % 32) is stored directly, and an output row length that is not a
    multiple of 4 floats takes the direct stores throughout."""
    torch = torch_cuda
    fmt = mgb.Q4_K
    w = synthetic.packed_weights(fmt, n, k, seed=m + n)
    x = synthetic.activations(m, k, seed=m)
    wdev = _device_layout(torch, fmt, w, n, k)
    y = _qmatmul(torch, fmt, wdev, n, k, x)
    assert np.isfinite(y).all()
    oracle.assert_close(y, oracle.packed_matmul(fmt, w, n, k, x), GEMM_TOL, f"gemm m {m} n {n}")


@pytest.mark.parametrize("m", [1, 2])
def test_gemv_chain_reads_the_previous_output(torch_cuda, oracle, m):
    """A decode chain: y1 = x W1^T then y2 = y1 W2^T on one stream, the second
    GEMV a programmatic dependent that starts while the first still writes y1,
    over three rounds with the same buffers (so earlier rounds have read y1's
    lines).  Every round equals the oracle chain: x is loaded coherently after
    the dependency wait, never through the read-only path."""
    torch = torch_cuda
    fmt, k, n1, n2 = mgb.Q4_K, 1024, 512, 256
    w1 = synthetic.packed_weights(fmt, n1, k, seed=91)
    w2 = synthetic.packed_weights(fmt, n2, n1, seed=92)
    d1, d2 = _device_layout(torch, fmt, w1, n1, k), _device_layout(torch, fmt, w2, n2, n1)
    xd = torch.empty((m, k), dtype=torch.float32, device="cuda")
    y1 = torch.empty((m, n1), dtype=torch.float32, device="cuda")
    y2 = torch.empty((m, n2), dtype=torch.float32, device="cuda")
    sp = torch.cuda.current_stream().cuda_stream
    for rnd in range(3):
        x = synthetic.activations(m, k, seed=93 + rnd)
        xd.copy_(torch.from_numpy(x))
        mgb.qmatmul(fmt, d1.data_ptr(), n1, k, xd.data_ptr(), m, y1.data_ptr(), stream=sp)
        mgb.qmatmul(fmt, d2.data_ptr(), n2, n1, y1.data_ptr(), m, y2.data_ptr(), stream=sp)
        torch.cuda.synchronize()
        assert mgb.take_device_error(torch.cuda.current_device()) == 0
        ref1 = oracle.packed_matmul(fmt, w1, n1, k, x)
        got1 = y1.cpu().numpy()
        oracle.assert_close(got1, ref1, GEMV_TOL, f"round {rnd} first")
        # the second GEMV against the oracle on the first's actual output
        oracle.assert_close(y2.cpu().numpy(), oracle.packed_matmul(fmt, w2, n2, n1, got1),
                            GEMV_TOL, f"round {rnd} second")
