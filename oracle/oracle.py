"""ctypes loader for the CPU oracle — TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may
import this module.  It checks (or, as the CPU baseline, is timed beside) the
B200 path; the product never routes through it.
"""

from __future__ import annotations

import ctypes
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle_mgb.so"
BASELINE_PATH = HERE / "_build" / "libcpu_baseline_mgb.so"

Q8_0, Q4_K, Q6_K, IQ4_NL, Q5_K, Q4_0 = 0, 1, 2, 5, 12, 13
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210), IQ4_NL: (32, 18), Q5_K: (256, 176),
         Q4_0: (32, 18)}

_lib = None
_baseline = None

_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u64 = ctypes.c_uint64


def build() -> None:
    """Compile the oracle and the CPU-baseline port with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        L.orc_f16_to_f32.restype = ctypes.c_float
        L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.orc_dequantize.argtypes = [ctypes.c_int, _u8p, _u64, _u64, _f32p]
        L.orc_matmul.argtypes = [_f32p, _u64, _u64, _f32p, _u64, _u64, ctypes.c_int,
                                 ctypes.c_int, _f32p]
        L.orc_packed_matmul.argtypes = [ctypes.c_int, _u8p, _u64, _u64, _f32p, _u64, _u64,
                                        ctypes.c_int, _f32p]
        L.orc_packed_axpy.argtypes = [ctypes.c_int, _u8p, _u64, _u64, _f32p, _u64, _u64, _f32p]
        L.orc_quantize_rows.argtypes = [_f32p, _u64, _i8p, _f32p, _i32p]
        L.orc_quantize_rows.restype = None
        L.orc_add.argtypes = [_f32p, _u64, _u64, _f32p, _u64, _f32p]
        L.orc_test_packed.argtypes = [ctypes.c_int, _u64, _u64, ctypes.c_uint32, _u8p]
        L.orc_test_packed.restype = None
        L.orc_test_activations.argtypes = [_u64, _u64, ctypes.c_uint32, _f32p]
        L.orc_test_activations.restype = None
        L.orc_iq4nl_values.restype = _i8p
        L.orc_q4_0_values.restype = _i8p
        L.orc_scale_min_k4.argtypes = [ctypes.c_int, _u8p, _u8p, _u8p]
        L.orc_scale_min_k4.restype = None
        _lib = L
    return _lib


def baseline() -> ctypes.CDLL:
    """The CPU-baseline port of the reference's default packed path (int8
    activations, AVX2 kernels, persistent pool; oracle/cpu_baseline.c)."""
    global _baseline
    if _baseline is None:
        if not BASELINE_PATH.exists():
            build()
        L = ctypes.CDLL(str(BASELINE_PATH))
        L.cpb_set_threads.argtypes = [ctypes.c_int]
        L.cpb_set_threads.restype = ctypes.c_int
        for name in ("cpb_packed_matmul", "cpb_packed_matmul_f32"):
            fn = getattr(L, name)
            fn.argtypes = [ctypes.c_int, _u8p, _u64, _u64, _f32p, _u64, _u64, _f32p]
            fn.restype = ctypes.c_int
        _baseline = L
    return _baseline


def baseline_packed_matmul(fmt: int, data: np.ndarray, stored_rows: int, stored_cols: int,
                           x: np.ndarray, int8: bool = True, threads: int = 1) -> np.ndarray:
    """Times the reference's own CPU path: y[m, stored_rows] (int8 activations by default)."""
    L = baseline()
    L.cpb_set_threads(threads)
    x = np.ascontiguousarray(x, dtype=np.float32)
    data = np.ascontiguousarray(data, dtype=np.uint8)
    m, k = x.shape
    y = np.empty((m, stored_rows), dtype=np.float32)
    fn = L.cpb_packed_matmul if int8 else L.cpb_packed_matmul_f32
    rc = fn(fmt, _p(data, _u8p), stored_rows, stored_cols, _p(x, _f32p), m, k, _p(y, _f32p))
    if rc:
        raise ValueError("cpu baseline: shape or format rejected")
    return y


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def row_bytes(fmt: int, cols: int) -> int:
    elems, bb = BLOCK[fmt]
    return cols // elems * bb


def dequantize(fmt: int, data: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """Stored-order f32 values of a packed matrix (`dequantize_row` per row)."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty((rows, cols), dtype=np.float32)
    rc = lib().orc_dequantize(fmt, _p(data, _u8p), rows, cols, _p(out, _f32p))
    if rc:
        raise ValueError(f"oracle cannot decode format {fmt}")
    return out


def matmul(a: np.ndarray, b: np.ndarray, transpose_a: bool = False,
           transpose_b: bool = False) -> np.ndarray:
    """The reference's correctness-first f32 matmul (src/lib.rs:262-318)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m = a.shape[1] if transpose_a else a.shape[0]
    n = b.shape[0] if transpose_b else b.shape[1]
    out = np.empty((m, n), dtype=np.float32)
    rc = lib().orc_matmul(_p(a, _f32p), a.shape[0], a.shape[1], _p(b, _f32p), b.shape[0],
                          b.shape[1], int(transpose_a), int(transpose_b), _p(out, _f32p))
    if rc:
        raise ValueError("matmul inner dimension mismatch")
    return out


def packed_matmul(fmt: int, data: np.ndarray, stored_rows: int, stored_cols: int,
                  x: np.ndarray, int8: bool = False) -> np.ndarray:
    """`NativeState::packed_matmul`: x[m,k] times W whose stored rows are the outputs."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    data = np.ascontiguousarray(data, dtype=np.uint8)
    m, k = x.shape
    y = np.empty((m, stored_rows), dtype=np.float32)
    rc = lib().orc_packed_matmul(fmt, _p(data, _u8p), stored_rows, stored_cols, _p(x, _f32p), m,
                                 k, int(int8), _p(y, _f32p))
    if rc:
        raise ValueError("packed matmul: shape or format rejected")
    return y


def packed_axpy(fmt: int, data: np.ndarray, stored_rows: int, stored_cols: int,
                x: np.ndarray) -> np.ndarray:
    """`axpy_columns`: W's stored rows are the k input rows; y[m, stored_cols]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    data = np.ascontiguousarray(data, dtype=np.uint8)
    m, k = x.shape
    y = np.empty((m, stored_cols), dtype=np.float32)
    rc = lib().orc_packed_axpy(fmt, _p(data, _u8p), stored_rows, stored_cols, _p(x, _f32p), m, k,
                               _p(y, _f32p))
    if rc:
        raise ValueError("packed axpy: shape or format rejected")
    return y


def quantize_rows(x: np.ndarray):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    n = x.size
    values = np.empty(n, dtype=np.int8)
    scales = np.empty(n // 32, dtype=np.float32)
    sums = np.empty((n // 32, 2), dtype=np.int32)
    lib().orc_quantize_rows(_p(x, _f32p), n, _p(values, _i8p), _p(scales, _f32p),
                            _p(sums, _i32p))
    return values, scales, sums


def int8_rounded(x: np.ndarray) -> np.ndarray:
    """The activations as int8 activations see them (src/native/tests.rs:77-89)."""
    values, scales, _ = quantize_rows(x)
    out = values.reshape(-1, 32).astype(np.float32) * scales[:, None]
    return out.reshape(x.shape).astype(np.float32)


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    rc = lib().orc_add(_p(a, _f32p), a.size, a.shape[-1], _p(b, _f32p), b.size, _p(out, _f32p))
    if rc:
        raise ValueError("add: shapes do not broadcast")
    return out


def test_packed(fmt: int, rows: int, cols: int, seed: int) -> np.ndarray:
    """The reference test generator `packed` (src/native/tests.rs:45-67)."""
    elems, bb = BLOCK[fmt]
    out = np.empty(rows * cols // elems * bb, dtype=np.uint8)
    lib().orc_test_packed(fmt, rows, cols, seed, _p(out, _u8p))
    return out


def test_activations(rows: int, cols: int, seed: int) -> np.ndarray:
    """The reference test generator `activations` (src/native/tests.rs:69-75)."""
    out = np.empty((rows, cols), dtype=np.float32)
    lib().orc_test_activations(rows, cols, seed, _p(out, _f32p))
    return out


def assert_close(actual: np.ndarray, expected: np.ndarray, tol: float, what: str = "") -> float:
    """The reference's tolerance rule (src/native/tests.rs:91-103):
    |a - e| <= tol * max(1, max|e|) for every element.  Returns the normalised
    max error."""
    assert actual.shape == expected.shape, (what, actual.shape, expected.shape)
    scale = max(1.0, float(np.max(np.abs(expected))) if expected.size else 1.0)
    err = float(np.max(np.abs(actual.astype(np.float64) - expected.astype(np.float64)))) \
        if expected.size else 0.0
    assert err <= tol * scale, f"{what}: max |a-e| {err} > {tol} * {scale}"
    return err / scale
