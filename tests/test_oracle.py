"""The CPU oracle, pinned before anything is checked against it.

- bit-exact against gguf-py 0.19.0's dequantisation (tests/golden/, made by
  tests/golden/make_golden.py), for reference-generator and random bytes;
- hand-built known-answer blocks;
- the reference's own conformance check (matmul 2x2, src/lib.rs:1882-1892);
- the reference's self-consistency tests restated (src/native/tests.rs).
"""

from __future__ import annotations

import pathlib
import struct

import numpy as np
import pytest

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "dequant_gguf.npz"
FORMAT_CODES = {"q8_0": 0, "q4_k": 1, "iq4_nl": 5, "q4_0": 13, "q6_k": 2, "q5_k": 12}


def _same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    nan = np.isnan(a)
    if not np.array_equal(nan, np.isnan(b)):
        return False
    return np.array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("name", sorted(FORMAT_CODES))
@pytest.mark.parametrize("source", ["reference_generator", "random_bytes"])
def test_dequant_matches_gguf_bit_exactly(oracle, name, source):
    golden = np.load(GOLDEN)
    key = f"{name}__{source}"
    code, rows, cols = (int(v) for v in golden[key + "__meta"])
    assert code == FORMAT_CODES[name]
    got = oracle.dequantize(code, golden[key + "__bytes"], rows, cols)
    assert _same_bits(got, golden[key + "__expected"]), f"{key} differs from gguf-py"


def test_codebook_matches_gguf(oracle):
    import ctypes

    golden = np.load(GOLDEN)
    table = np.ctypeslib.as_array(oracle.lib().orc_iq4nl_values(), shape=(16,)).copy()
    assert np.array_equal(table, golden["iq4_nl_kvalues"])
    q40 = np.ctypeslib.as_array(oracle.lib().orc_q4_0_values(), shape=(16,)).copy()
    assert np.array_equal(q40, np.arange(16, dtype=np.int8) - 8)
    assert ctypes.sizeof(ctypes.c_int8) == 1


def test_f16_conversion_is_exact_for_every_pattern(oracle):
    bits = np.arange(65536, dtype=np.uint16)
    expected = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.lib().orc_f16_to_f32(int(b)) for b in bits[::7]], dtype=np.float32)
    assert _same_bits(got, expected[::7])


def _f16(v: float) -> bytes:
    return struct.pack("<e", v)


def test_q4k_known_answer(oracle):
    # d = 0.5, dmin = 0.25; sub-block j scale = j + 1, min = 2j (all < 16, so the
    # high-bit packing is exercised by j >= 4 through the 12-byte layout).
    sc = [j + 1 for j in range(8)]
    mn = [2 * j for j in range(8)]
    scales = bytearray(12)
    for j in range(4):
        scales[j] = sc[j] | ((sc[j + 4] >> 4) << 6)
        scales[j + 4] = mn[j] | ((mn[j + 4] >> 4) << 6)
        scales[j + 8] = (sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4)
    qs = bytes(((i % 16) | (((i + 3) % 16) << 4)) for i in range(128))
    block = _f16(0.5) + _f16(0.25) + bytes(scales) + qs
    got = oracle.dequantize(1, np.frombuffer(block, dtype=np.uint8), 1, 256)[0]
    expected = []
    for j in range(8):
        chunk = qs[32 * (j // 2): 32 * (j // 2) + 32]
        for byte in chunk:
            q = (byte >> (4 * (j % 2))) & 0xF
            expected.append(np.float32(0.5 * sc[j]) * np.float32(q) - np.float32(0.25 * mn[j]))
    assert np.array_equal(got, np.array(expected, dtype=np.float32))


def test_q4k_six_bit_scales_known_answer(oracle):
    # scale 63 / min 33 in sub-blocks 4..7 need the two high bits packed in bytes 0..7
    scales = bytearray(12)
    for j in range(4):
        scales[j] = 5 | ((63 >> 4) << 6)
        scales[j + 4] = 7 | ((33 >> 4) << 6)
        scales[j + 8] = (63 & 0xF) | ((33 & 0xF) << 4)
    block = _f16(1.0) + _f16(1.0) + bytes(scales) + bytes([0x21] * 128)
    got = oracle.dequantize(1, np.frombuffer(block, dtype=np.uint8), 1, 256)[0]
    assert np.all(got[:32] == 5 * 1 - 7) and np.all(got[32:64] == 5 * 2 - 7)
    assert np.all(got[128:160] == 63 * 1 - 33) and np.all(got[160:192] == 63 * 2 - 33)


def test_q6k_known_answer(oracle):
    # q code c (0..63) of value i of the block = (i * 7) % 64, so every code
    # appears; scales s_t = t - 8 (negative, zero and positive int8), d = 0.25.
    codes = [(i * 7) % 64 for i in range(256)]
    ql, qh = bytearray(128), bytearray(64)
    for run in range(8):
        h, g = run // 4, run % 4
        for i in range(32):
            c = codes[32 * run + i]
            ql[64 * h + 32 * (g % 2) + i] |= (c & 0xF) << (4 * (g // 2))
            qh[32 * h + i] |= (c >> 4) << (2 * g)
    scales = bytes((t - 8) & 0xFF for t in range(16))
    block = bytes(ql) + bytes(qh) + scales + _f16(0.25)
    got = oracle.dequantize(2, np.frombuffer(block, dtype=np.uint8), 1, 256)[0]
    expected = [np.float32(np.float32(0.25) * np.float32(i // 16 - 8)) * np.float32(codes[i] - 32)
                for i in range(256)]
    assert np.array_equal(got, np.array(expected, dtype=np.float32))


def test_q5k_known_answer(oracle):
    # 5-bit codes (i * 5) % 32; Q4_K's scale layout (scale j + 1, min j, < 16)
    codes = [(i * 5) % 32 for i in range(256)]
    qh, ql = bytearray(32), bytearray(128)
    for run in range(8):
        for i in range(32):
            c = codes[32 * run + i]
            ql[32 * (run // 2) + i] |= (c & 0xF) << (4 * (run % 2))
            qh[i] |= (c >> 4) << run
    scales = bytearray(12)
    for j in range(4):
        scales[j] = j + 1
        scales[j + 4] = j
        scales[j + 8] = (j + 5) | ((j + 4) << 4)
    block = _f16(0.5) + _f16(0.125) + bytes(scales) + bytes(qh) + bytes(ql)
    got = oracle.dequantize(12, np.frombuffer(block, dtype=np.uint8), 1, 256)[0]
    expected = [np.float32(0.5 * (i // 32 + 1)) * np.float32(codes[i]) - np.float32(0.125 * (i // 32))
                for i in range(256)]
    assert np.array_equal(got, np.array(expected, dtype=np.float32))


def test_q8_0_and_iq4_known_answers(oracle):
    q = np.arange(-16, 16, dtype=np.int8)
    block = _f16(0.125) + q.tobytes()
    got = oracle.dequantize(0, np.frombuffer(block, dtype=np.uint8), 1, 32)[0]
    assert np.array_equal(got, q.astype(np.float32) * np.float32(0.125))
    idx = bytes((i | ((15 - i) << 4)) for i in range(16))
    block = _f16(-2.0) + idx
    table = np.array([-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113],
                     dtype=np.float32)
    got = oracle.dequantize(5, np.frombuffer(block, dtype=np.uint8), 1, 32)[0]
    expected = np.concatenate([table[np.arange(16)], table[15 - np.arange(16)]]) * -2.0
    assert np.array_equal(got, expected.astype(np.float32))
    got = oracle.dequantize(13, np.frombuffer(block, dtype=np.uint8), 1, 32)[0]
    expected = np.concatenate([np.arange(16) - 8, (15 - np.arange(16)) - 8]) * -2.0
    assert np.array_equal(got, expected.astype(np.float32))


def test_conformance_matmul_2x2(oracle):
    # src/lib.rs:1882-1892: [[1,2],[3,4]] x [[5,6],[7,8]] = [19,22,43,50]
    a = np.array([[1, 2], [3, 4]], dtype=np.float32)
    b = np.array([[5, 6], [7, 8]], dtype=np.float32)
    assert oracle.matmul(a, b).reshape(-1).tolist() == [19, 22, 43, 50]
    assert oracle.matmul(a, b, True, False).tolist() == (a.T @ b).tolist()
    assert oracle.matmul(a, b, False, True).tolist() == (a @ b.T).tolist()


def test_matmul_propagates_nan_through_zero(oracle):
    # src/tests.rs:115-128: 0 * NaN must stay NaN (no zero-skip)
    a = np.array([[0.0, 1.0]], dtype=np.float32)
    b = np.array([[np.nan], [2.0]], dtype=np.float32)
    assert np.isnan(oracle.matmul(a, b)[0, 0])


@pytest.mark.parametrize("fmt", [0, 1, 2, 5, 12, 13])
def test_packed_matmul_equals_dense_reference(oracle, fmt):
    # src/native/tests.rs:134-154 restated: f32 activations are bit-identical to
    # the dense oracle (same per-element values, same sequential order), int8
    # activations match the dense matmul of the int8-rounded activations.
    k, n = 512, 37
    w = oracle.test_packed(fmt, n, k, 21)
    dense = oracle.dequantize(fmt, w, n, k)  # stored [n, k] = logical [k, n] transposed
    for m in (1, 3, 9):
        a = oracle.test_activations(m, k, m)
        expected = oracle.matmul(a, dense, False, True)
        got = oracle.packed_matmul(fmt, w, n, k, a)
        assert np.array_equal(got, expected)
        got8 = oracle.packed_matmul(fmt, w, n, k, a, int8=True)
        expected8 = oracle.matmul(oracle.int8_rounded(a), dense, False, True)
        oracle.assert_close(got8, expected8, 2e-5, f"fmt {fmt} int8 m {m}")


@pytest.mark.parametrize("fmt", [0, 5, 13])
def test_odd_run_counts(oracle, fmt):
    # src/native/tests.rs:156-174
    k, n = 96, 5
    w = oracle.test_packed(fmt, n, k, 23)
    dense = oracle.dequantize(fmt, w, n, k)
    a = oracle.test_activations(2, k, 7)
    oracle.assert_close(oracle.packed_matmul(fmt, w, n, k, a, int8=True),
                        oracle.matmul(oracle.int8_rounded(a), dense, False, True), 2e-5)


@pytest.mark.parametrize("fmt", [0, 1, 2, 5, 12, 13])
def test_input_major_axpy(oracle, fmt):
    # src/native/tests.rs:194-210: stored rows = input rows
    w = oracle.test_packed(fmt, 64, 256, 61)
    dense = oracle.dequantize(fmt, w, 64, 256)  # logical [64, 256]
    for m in (1, 4):
        a = oracle.test_activations(m, 64, 62)
        oracle.assert_close(oracle.packed_axpy(fmt, w, 64, 256, a), oracle.matmul(a, dense),
                            2e-5, f"axpy {fmt}")


def test_shape_errors_are_reported(oracle):
    w = oracle.test_packed(1, 4, 256, 1)
    with pytest.raises(ValueError):
        oracle.packed_matmul(1, w, 4, 256, np.zeros((1, 128), np.float32))
    with pytest.raises(ValueError):
        oracle.dequantize(3, w, 1, 256)  # Q2_K is declined by this oracle


def test_bias_broadcast(oracle):
    a = np.arange(6, dtype=np.float32).reshape(2, 3)
    b = np.array([10, 20, 30], dtype=np.float32)
    assert oracle.add(a, b).tolist() == [[10, 21, 32], [13, 24, 35]]
    with pytest.raises(ValueError):
        oracle.add(a, np.ones(4, np.float32))


@pytest.mark.parametrize("fmt", [0, 1, 5, 13])
@pytest.mark.parametrize("threads", [1, 4])
def test_cpu_baseline_port_matches_the_oracle(oracle, fmt, threads):
    # the timed CPU arm (AVX2 restatement + pool) agrees with the scalar oracle
    # the way the reference's own test does (src/native/tests.rs:134-154)
    k, n = 512, 37
    w = oracle.test_packed(fmt, n, k, 21)
    dense = oracle.dequantize(fmt, w, n, k)
    for m in (1, 3, 9):
        a = oracle.test_activations(m, k, m)
        got = oracle.baseline_packed_matmul(fmt, w, n, k, a, int8=True, threads=threads)
        oracle.assert_close(got, oracle.matmul(oracle.int8_rounded(a), dense, False, True), 2e-5)
        got32 = oracle.baseline_packed_matmul(fmt, w, n, k, a, int8=False, threads=threads)
        assert np.array_equal(got32, oracle.matmul(a, dense, False, True))
    if fmt != 1:  # odd run counts take the paired kernels' tail (src/native/tests.rs:156-174)
        w = oracle.test_packed(fmt, 5, 96, 23)
        a = oracle.test_activations(2, 96, 7)
        oracle.assert_close(oracle.baseline_packed_matmul(fmt, w, 5, 96, a, threads=threads),
                            oracle.packed_matmul(fmt, w, 5, 96, a, int8=True), 2e-5)


def quantize_edge_rows() -> np.ndarray:
    """Activation blocks that probe `quantize_rows` (src/native/quant.rs:350-378):
    N(0, 1) rows, an all-zero block, exact ties at .5 (amax 127 makes d = 1),
    +-amax at both ends, a NaN and an infinity (amax then ignores the NaN, and
    inf / inf is NaN, which `as i8` maps to 0)."""
    rng = np.random.default_rng(0x5EED)
    blocks = [rng.standard_normal(32 * 64, dtype=np.float32).reshape(-1, 32)]
    blocks.append(np.zeros((1, 32), np.float32))
    ties = np.array([127.0, -127.0, 2.5, 3.5, -2.5, -3.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5]
                    + [4.5] * 20, np.float32)
    blocks.append(ties[None])
    amax = rng.standard_normal(32).astype(np.float32)
    amax[0], amax[31] = 7.25, -7.25
    blocks.append(amax[None])
    nan = rng.standard_normal(32).astype(np.float32)
    nan[5] = np.nan
    blocks.append(nan[None])
    inf = rng.standard_normal(32).astype(np.float32)
    inf[9] = np.inf
    blocks.append(inf[None])
    tiny = np.full((1, 32), 1e-30, np.float32)
    tiny[0, 3] = -3e-38
    blocks.append(tiny)
    return np.concatenate(blocks).reshape(-1)


def test_quantize_rows_known_answers(oracle):
    values, scales, sums = oracle.quantize_rows(quantize_edge_rows())
    v = values.reshape(-1, 32)
    z, t, nan, inf = 64, 65, 67, 68
    assert not v[z].any() and scales[z] == 0.0 and not sums[z].any()
    assert scales[t] == 1.0
    # round half to even, division (not a reciprocal) by d = amax / 127
    assert list(v[t, :12]) == [127, -127, 2, 4, -2, -4, 0, 0, 2, -2, 126, -126]
    assert list(sums[t]) == [int(v[t, :16].sum()), int(v[t, 16:].sum())]
    assert v[66, 0] == 127 and v[66, 31] == -127
    assert v[nan, 5] == 0 and np.isfinite(scales[nan])
    assert scales[inf] == np.inf and v[inf, 9] == 0 and not v[inf].any()
