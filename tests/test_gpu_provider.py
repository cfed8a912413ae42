"""The Provider contract on the GPU, ported from the reference's executor
tests (src/native/tests.rs) onto the C ABI, plus the error paths of
`submit_kernel` / `complete_kernel` (src/lib.rs:2301-2404)."""

from __future__ import annotations

import numpy as np
import pytest

import magnetar_b200 as mgb

pytestmark = pytest.mark.gpu
FORMATS = [mgb.Q4_K, mgb.Q5_K, mgb.Q6_K, mgb.Q8_0, mgb.IQ4_NL, mgb.Q4_0]


@pytest.fixture()
def provider(cuda_device):
    p = mgb.B200Provider(device=cuda_device)
    yield p
    p.close()


def _tol(m):
    return 1e-3 if m <= 2 else 5e-3


def test_executor_stores_packed_weights(provider, oracle):
    # src/native/tests.rs:251-274
    w = oracle.test_packed(mgb.Q4_K, 4, 256, 41)
    assert provider.write_packed_weight_tensor("w", mgb.Q4_K, 4, 256, True, w) == "Stored"
    assert provider.is_packed("w")
    stored = oracle.dequantize(mgb.Q4_K, w, 4, 256)
    got = provider.read_tensor("w")
    assert got.shape == (256, 4)
    assert np.array_equal(got, stored.T)  # logical [k, n] of a transposed weight, bit-exact
    assert provider.resident_shape("w") == [256, 4]
    assert provider.materializations() == 1
    assert provider.release_tensor("w")
    assert not provider.is_packed("w")
    assert not provider.release_tensor("w")
    with mgb.B200Provider(packed_weights=False) as declining:
        assert declining.write_packed_weight_tensor("w", mgb.Q4_K, 4, 256, True, w) == "Declined"
    # a format this Provider does not execute is declined (the Runtime loads f32)
    assert provider.write_packed_weight_tensor("q2", 3, 1, 256, True,  # Q2_K
                                               np.zeros(84, np.uint8)) == "Declined"


def test_packed_weights_survive_opaque_writes_and_yield_to_copies(provider, oracle):
    # src/native/tests.rs:276-313
    w = oracle.test_packed(mgb.Q8_0, 2, 32, 43)
    provider.write_packed_weight_tensor("w", mgb.Q8_0, 2, 32, True, w)
    assert provider.read_tensor_value("w") == "Opaque"
    provider.write_tensor_value_opaque("w")
    assert provider.is_packed("w")
    replacement = np.full((32, 2), 0.5, dtype=np.float32)
    provider.write_tensor("source", replacement)
    provider.copy_tensor("source", "w")
    assert not provider.is_packed("w")
    assert np.array_equal(provider.read_tensor("w"), replacement)
    assert provider.read_tensor_value("nothing") is None


def test_write_tensor_forgets_packed(provider, oracle):
    w = oracle.test_packed(mgb.Q8_0, 2, 32, 1)
    provider.write_packed_weight_tensor("w", mgb.Q8_0, 2, 32, True, w)
    provider.write_tensor("w", np.ones((3, 3), np.float32))
    assert not provider.is_packed("w")
    assert provider.resident_shape("w") == [3, 3]


@pytest.mark.parametrize("fmt", FORMATS)
def test_packed_matmuls_match_the_reference_cpu(provider, oracle, fmt):
    # src/native/tests.rs:134-154 (k = 512, n = 37, m in {1, 3, 9}), f32 and int8 activations
    k, n = 512, 37
    w = oracle.test_packed(fmt, n, k, 21)
    dense = oracle.dequantize(fmt, w, n, k)
    provider.write_packed_weight_tensor("w", fmt, n, k, True, w)
    with mgb.B200Provider(int8_activations=True) as p8:
        p8.write_packed_weight_tensor("w", fmt, n, k, True, w)
        for m in (1, 3, 9):
            a = oracle.test_activations(m, k, m)
            expected = oracle.matmul(a, dense, False, True)
            oracle.assert_close(provider.matmul(a, "w"), expected, _tol(m), f"fmt {fmt} m {m}")
            expected8 = oracle.matmul(oracle.int8_rounded(a), dense, False, True)
            oracle.assert_close(p8.matmul(a, "w"), expected8, _tol(m), f"fmt {fmt} int8 m {m}")


@pytest.mark.parametrize("fmt", [mgb.Q8_0, mgb.IQ4_NL, mgb.Q4_0])
def test_odd_run_counts(provider, oracle, fmt):
    # src/native/tests.rs:156-174: k = 96 holds an odd number of runs
    k, n = 96, 5
    w = oracle.test_packed(fmt, n, k, 23)
    provider.write_packed_weight_tensor("w", fmt, n, k, True, w)
    for m in (2, 5):
        a = oracle.test_activations(m, k, 7)
        oracle.assert_close(provider.matmul(a, "w"), oracle.packed_matmul(fmt, w, n, k, a), 1e-3)


def test_tied_head_reads_an_untransposed_table_packed(provider, oracle):
    # src/native/tests.rs:176-192: a [50, 64] table used with transpose_b
    table = oracle.test_packed(mgb.Q8_0, 50, 64, 31)
    dense = oracle.dequantize(mgb.Q8_0, table, 50, 64)
    provider.write_packed_weight_tensor("t", mgb.Q8_0, 50, 64, False, table)
    assert np.array_equal(provider.read_tensor("t"), dense)
    a = oracle.test_activations(2, 64, 3)
    got = provider.matmul(a, "t", transpose_b=True)
    oracle.assert_close(got, oracle.matmul(a, dense, False, True), 1e-3)


@pytest.mark.parametrize("fmt", FORMATS)
def test_input_major_weights_multiply_packed(provider, oracle, fmt):
    # src/native/tests.rs:194-210: stored rows are the input rows
    w = oracle.test_packed(fmt, 64, 256, 61)
    dense = oracle.dequantize(fmt, w, 64, 256)
    provider.write_packed_weight_tensor("w", fmt, 64, 256, False, w)
    for m in (1, 4):
        a = oracle.test_activations(m, 64, 62)
        oracle.assert_close(provider.matmul(a, "w"), oracle.matmul(a, dense), 2e-5)


def test_transpose_a_expands_the_weight(provider, oracle):
    w = oracle.test_packed(mgb.Q4_K, 8, 256, 5)
    dense = oracle.dequantize(mgb.Q4_K, w, 8, 256)  # stored [8, 256]; logical [256, 8]
    provider.write_packed_weight_tensor("w", mgb.Q4_K, 8, 256, True, w)
    a = oracle.test_activations(256, 3, 4)  # used transposed: [3, 256]
    got = provider.matmul(a, "w", transpose_a=True)
    oracle.assert_close(got, oracle.matmul(a, dense.T.copy(), True, False), 1e-4)
    assert provider.materializations() >= 1


def test_f32_weight_runs_the_dense_kernel(provider, oracle):
    b = oracle.test_activations(64, 48, 2)
    provider.write_tensor("b", b)
    a = oracle.test_activations(5, 64, 3)
    oracle.assert_close(provider.matmul(a, "b"), oracle.matmul(a, b), 1e-5)
    oracle.assert_close(provider.matmul(a[:, :48].copy(), "b", transpose_b=True),
                        oracle.matmul(a[:, :48].copy(), b, False, True), 1e-5)


@pytest.mark.parametrize("m", [1, 16])
def test_bias_and_residual_kernels(provider, oracle, m):
    fmt, k, n = mgb.Q4_K, 512, 40
    w = oracle.test_packed(fmt, n, k, 8)
    provider.write_packed_weight_tensor("w", fmt, n, k, True, w)
    a = oracle.test_activations(m, k, 2)
    base = oracle.packed_matmul(fmt, w, n, k, a)
    provider.write_tensor("a", a)
    bias = np.linspace(-1, 1, n, dtype=np.float32)
    provider.write_tensor("bias", bias)
    h = provider.submit_kernel("matmul-bias", ["a", "w", "bias"], "y")
    assert provider.complete_kernel(h).ok
    oracle.assert_close(provider.read_tensor("y"), oracle.add(base, bias), _tol(m))
    resid = oracle.test_activations(m, n, 3)
    provider.write_tensor("r", resid)
    h = provider.submit_kernel("matmul-residual", ["a", "w", "r"], "y")
    assert provider.complete_kernel(h).ok
    oracle.assert_close(provider.read_tensor("y"), oracle.add(resid, base), _tol(m))


def test_kernel_errors_and_single_consumption(provider, oracle):
    w = oracle.test_packed(mgb.Q4_K, 4, 256, 1)
    provider.write_packed_weight_tensor("w", mgb.Q4_K, 4, 256, True, w)
    provider.write_tensor("x", np.ones((1, 256), np.float32))
    # deadline already elapsed (src/lib.rs:2372-2380)
    h = provider.submit_kernel("matmul", ["x", "w"], "y", deadline_ms=0)
    assert provider.complete_kernel(h).status == mgb.TIMEOUT
    # single consumption (src/lib.rs:2337-2356)
    h = provider.submit_kernel("matmul", ["x", "w"], "y")
    assert provider.complete_kernel(h).ok
    with pytest.raises(mgb.MgbError) as info:
        provider.complete_kernel(h)
    assert info.value.status == mgb.UNKNOWN_HANDLE
    # accumulation dtype other than f32 (src/lib.rs:2445-2456)
    h = provider.submit_kernel("matmul", ["x", "w"], "y", accumulation_dtype=2)
    assert provider.complete_kernel(h).status == mgb.DTYPE_UNSUPPORTED
    # an unknown kernel, a missing input, a shape mismatch (src/native/mod.rs:118-125)
    assert provider.complete_kernel(provider.submit_kernel("rope", ["x"], "y")).status == \
        mgb.KERNEL_NOT_FOUND
    r = provider.complete_kernel(provider.submit_kernel("matmul", ["nope", "w"], "y"))
    assert r.status == mgb.EXECUTION_FAILED and "no materialized data" in r.reason
    provider.write_tensor("x2", np.ones((1, 128), np.float32))
    r = provider.complete_kernel(provider.submit_kernel("matmul", ["x2", "w"], "y"))
    assert r.status == mgb.EXECUTION_FAILED
    assert "activations have 128 columns, the weight's stored rows 256" in r.reason
    kinds = [o["kind"] for o in provider.observations()]
    assert kinds.count(2) >= 6 and 5 in kinds and 4 in kinds and 3 in kinds


def test_identity_device_and_observations(provider):
    provider.initialize()
    obs = provider.observations()
    assert [o["kind"] for o in obs[:2]] == [0, 1]
    assert "b200-native" in obs[0]["detail"]
    d = provider.device()
    assert d["architecture"].startswith("sm_10") and d["compute_units"] >= 100
    assert provider.health() == 0
    free, total = provider.device_memory()
    assert 0 < free <= total


def test_invalid_packed_bytes_are_rejected(provider):
    with pytest.raises(mgb.MgbError) as info:
        provider.write_packed_weight_tensor("w", mgb.Q4_K, 4, 256, True, np.zeros(10, np.uint8))
    assert info.value.status == mgb.INVALID_ARGUMENT
    with pytest.raises(mgb.MgbError):
        provider.write_packed_weight_tensor("w", mgb.Q4_K, 4, 100, True, np.zeros(10, np.uint8))


def test_calls_from_several_threads(provider, oracle):
    """The reference's Provider methods take `&self` (src/native/mod.rs:565-700):
    several threads may drive one Provider.  Uploads and downloads overlap
    other threads' calls here; every thread must still get its own result."""
    import threading

    n, k, m = 512, 1024, 64
    w = oracle.test_packed(mgb.Q4_K, n, k, 7)
    provider.write_packed_weight_tensor("w", mgb.Q4_K, n, k, True, w)
    rng = np.random.default_rng(3)
    xs = [rng.standard_normal((m, k)).astype(np.float32) for _ in range(4)]
    expect = []
    for t, x in enumerate(xs):  # one thread first: the results to reproduce
        provider.write_tensor(f"x{t}", x)
        assert provider.complete_kernel(provider.submit_kernel("matmul", [f"x{t}", "w"], f"y{t}")).ok
        expect.append(provider.read_tensor(f"y{t}"))
    oracle.assert_close(expect[0], oracle.packed_matmul(mgb.Q4_K, w, n, k, xs[0]), _tol(m), "y0")
    errors: list[str] = []

    def lane(t: int) -> None:
        for i in range(12):
            provider.write_tensor(f"x{t}", xs[t])
            r = provider.complete_kernel(provider.submit_kernel("matmul", [f"x{t}", "w"], f"y{t}"))
            y = provider.read_tensor(f"y{t}")
            if not r.ok or not np.array_equal(y, expect[t]):
                errors.append(f"thread {t} step {i}: {r.reason or 'wrong values'}")

    threads = [threading.Thread(target=lane, args=(t,)) for t in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert not errors, errors


def test_release_and_overwrite_during_a_download(provider):
    """A download reads its buffer with the Provider's mutex released: a
    release or an overwrite of the same resource meanwhile must neither free
    the buffer under the copy nor tear the values read."""
    import threading

    big = np.arange(16 << 20, dtype=np.float32).reshape(4096, 4096)  # 64 MiB
    other = np.full_like(big, -1.0)
    outcomes: list[str] = []
    for trial in range(6):
        provider.write_tensor("t", big)
        got: list[object] = []

        def reader() -> None:
            try:
                got.append(provider.read_tensor("t"))
            except mgb.MgbError as e:
                got.append(e.status)

        th = threading.Thread(target=reader)
        th.start()
        if trial % 2:
            provider.release_tensor("t")
        else:
            provider.write_tensor("t", other)
        th.join()
        v = got[0]
        if isinstance(v, np.ndarray):
            assert np.array_equal(v, big) or np.array_equal(v, other), f"trial {trial}: torn read"
            outcomes.append("old" if np.array_equal(v, big) else "new")
        else:
            assert v == mgb.NOT_FOUND or v is None
            outcomes.append("gone")
    assert len(outcomes) == 6


@pytest.mark.parametrize("fmt", [mgb.Q4_K, mgb.Q8_0])
def test_zero_rows_and_large_k(provider, oracle, fmt):
    """An activation of zero rows gives a [0, N] output, as the reference's
    packed_matmul does for an empty batch (src/native/mod.rs:109-152); and a
    K past 1,024 runs (a 405B-class down projection) is served, not refused."""
    n, k = 16, 40960
    w = oracle.test_packed(fmt, n, k, 31)
    provider.write_packed_weight_tensor("w", fmt, n, k, True, w)
    y0 = provider.matmul(np.zeros((0, k), np.float32), "w")
    assert y0.shape == (0, n)
    x = oracle.test_activations(2, k, 7)
    oracle.assert_close(provider.matmul(x, "w"), oracle.packed_matmul(fmt, w, n, k, x), 1e-3,
                        f"fmt {fmt} k {k}")
