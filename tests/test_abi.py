"""The C-ABI library on the CPU-only container: it loads, exports every
function include/magnetar_b200.h declares, answers the identity queries and
fails cleanly (no crash, a status and a reason) where a GPU is needed."""

from __future__ import annotations

import ctypes

import pytest

import magnetar_b200 as mgb


def test_library_exports_every_header_function():
    lib = mgb.lib()
    declared = mgb.header_functions()
    assert len(declared) >= 35, declared
    missing = [f for f in declared if not hasattr(lib, f)]
    assert not missing, missing
    # and the Python mirror binds exactly what the header declares
    assert sorted(mgb._SIGNATURES) == declared


def test_identity_and_advertisements():
    assert mgb.lib().mgb_abi_version() == 3
    md = mgb.metadata()
    assert md["name"] == "magnetar:provider/b200-native"
    assert md["name"] != "magnetar:provider/reference-cpu"
    ads = mgb.kernel_advertisements()
    assert [a["name"] for a in ads] == ["matmul", "matmul-bias", "matmul-residual", "embedding"]
    assert all(a["rank"] == 2 and a["cancellation"] == 1 for a in ads)


def test_status_names_and_packed_sizes():
    assert mgb.status_name(mgb.DECLINED) == "declined"
    assert mgb.status_name(mgb.TIMEOUT) == "kernel-timeout"
    # device layout bytes equal the ggml block bytes
    assert mgb.packed_bytes(mgb.Q4_K, 4096, 4096) == 9_437_184
    assert mgb.packed_bytes(mgb.Q8_0, 14336, 4096) == 62_390_272
    assert mgb.packed_bytes(mgb.IQ4_NL, 14336, 4096) == 33_030_144
    assert mgb.packed_bytes(mgb.Q6_K, 14336, 4096) == 14336 * 16 * 224  # padded header
    assert mgb.packed_bytes(mgb.Q5_K, 14336, 4096) == 14336 * 16 * 176
    assert mgb.packed_bytes(3, 1, 256) == 0  # Q2_K: declined format
    # decode GEMV: no scratch; prefill GEMM: the bf16 activations
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 1, 4096, 4096) == 0
    assert mgb.qmatmul_workspace_bytes(mgb.Q8_0, 2, 14336, 4096) == 0
    assert mgb.qmatmul_workspace_bytes(mgb.Q8_0, 3, 5, 96) == 0  # ragged k: GEMV pairs
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 512, 14336, 4096) == 512 * 4096 * 2
    # m <= 128: room for the split-K partial planes too (K parts per tile)
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 64, 4096, 4096) == 64 * 4096 * 2 + 4 * 64 * 4096 * 4
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 64, 8192, 4096) == 64 * 4096 * 2 + 2 * 64 * 8192 * 4
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 64, 14336, 4096) == 64 * 4096 * 2  # wide tiles
    assert mgb.qmatmul_min_workspace_bytes(mgb.Q4_K, 64, 4096, 4096) == 64 * 4096 * 2
    # 129..512 rows (256-row tiles): split where the unsplit tiles would be narrow
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 130, 4096, 4096) == \
        130 * 4096 * 2 + 4 * 130 * 4096 * 4
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 512, 3584, 4096) == 512 * 4096 * 2
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 600, 1024, 8192) == \
        600 * 8192 * 2 + 4 * 600 * 1024 * 4
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 2048, 3584, 8192) == 2048 * 8192 * 2  # wide tiles
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 2048, 128, 8192) == \
        2048 * 8192 * 2 + 8 * 2048 * 128 * 4  # a sparse grid of narrow tiles
    assert mgb.qmatmul_workspace_bytes(mgb.Q4_K, 64, 512, 256 * 3) == 64 * 768 * 2  # k % 512
    assert mgb.qmatmul_min_workspace_bytes(mgb.Q4_K, 2, 512, 4096) == 0


def test_settings_from_env(monkeypatch):
    monkeypatch.setenv("MAGNETAR_B200_PACKED_WEIGHTS", "0")
    monkeypatch.setenv("MAGNETAR_B200_INT8_ACTIVATIONS", "1")
    monkeypatch.setenv("MAGNETAR_B200_KERNEL", "gemm")
    monkeypatch.setenv("MAGNETAR_B200_DEVICE", "3")
    s = mgb.settings_from_env()
    assert (s.packed_weights, s.int8_activations, s.kernel, s.device) == (0, 1, mgb.KERNEL_GEMM, 3)
    monkeypatch.delenv("MAGNETAR_B200_PACKED_WEIGHTS")
    monkeypatch.delenv("MAGNETAR_B200_INT8_ACTIVATIONS")
    monkeypatch.delenv("MAGNETAR_B200_KERNEL")
    s = mgb.settings_from_env()
    assert (s.packed_weights, s.int8_activations, s.kernel) == (1, 0, mgb.KERNEL_AUTO)


def test_provider_create_fails_cleanly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(mgb.MgbError) as info:
        mgb.B200Provider()
    assert info.value.status == mgb.CUDA_ERROR
    assert "CUDA device" in str(info.value)


def test_null_arguments_are_rejected_without_device_work():
    lib = mgb.lib()
    assert lib.mgb_provider_create(None, None) == mgb.INVALID_ARGUMENT
    assert lib.mgb_take_device_error(0, None) == mgb.INVALID_ARGUMENT
    assert lib.mgb_kernel_advertisement_get(99, ctypes.byref(mgb.Advertisement())) == \
        mgb.INVALID_ARGUMENT
    # a format the Provider does not execute, or a ragged shape, is refused up front
    assert lib.mgb_qmatmul(3, None, 1, 256, None, 1, None, None, 0, None, 0, None) == \
        mgb.UNSUPPORTED
    assert lib.mgb_qmatmul(mgb.Q4_K, None, 1, 96, None, 1, None, None, 0, None, 0, None) == \
        mgb.EXECUTION_FAILED
    assert "activations have 96 columns" in mgb.last_error()


def test_tensor_parallel_outputs_are_checked_before_device_work():
    lib = mgb.lib()
    fake = 1 << 40  # never dereferenced: every case fails validation first
    good = mgb.tp_out([fake, fake], [fake, fake], fake, ldy=512, col0=256, epoch=1, rank=1)

    def call(out):
        return lib.mgb_qmatmul_tp(mgb.Q4_K, fake, 256, 256, fake, 1, ctypes.byref(out), None, 0,
                                  None, 0, None)

    bad = mgb.tp_out([fake] * 2, [fake] * 2, fake, ldy=512, col0=256, epoch=1, rank=2)
    assert call(bad) == mgb.INVALID_ARGUMENT and "rank 2 of world 2" in mgb.last_error()
    bad = mgb.tp_out([fake] * 2, [fake] * 2, 0, ldy=512, col0=256, epoch=1, rank=1)
    assert call(bad) == mgb.INVALID_ARGUMENT and "CTA counter" in mgb.last_error()
    bad = mgb.tp_out([fake] * 2, [fake] * 2, fake, ldy=500, col0=256, epoch=1, rank=1)
    assert call(bad) == mgb.INVALID_ARGUMENT and "exceed the output row" in mgb.last_error()
    bad = mgb.tp_out([fake, 0], [fake] * 2, fake, ldy=512, col0=256, epoch=1, rank=1)
    assert call(bad) == mgb.INVALID_ARGUMENT and "rank 1" in mgb.last_error()
    with pytest.raises(ValueError):
        mgb.tp_out([fake] * 2, [fake], fake, ldy=512, col0=0, epoch=1, rank=0)
    nine = mgb.TpOut()
    nine.world, nine.rank, nine.cta_counter = 9, 0, fake
    assert call(nine) == mgb.INVALID_ARGUMENT
    assert lib.mgb_qmatmul_tp(mgb.Q4_K, fake, 256, 256, fake, 1, None, None, 0, None, 0, None) \
        == mgb.INVALID_ARGUMENT
    # the shape checks of mgb_qmatmul apply to the shard
    assert lib.mgb_qmatmul_tp(mgb.Q4_K, fake, 256, 96, fake, 1, ctypes.byref(good), None, 0, None,
                              0, None) == mgb.EXECUTION_FAILED
    assert lib.mgb_tp_wait(None, 2, 1, 0, None) == mgb.INVALID_ARGUMENT
    assert lib.mgb_tp_wait(fake, 0, 1, 0, None) == mgb.INVALID_ARGUMENT
    assert lib.mgb_ipc_open(None, None) == mgb.INVALID_ARGUMENT
    assert lib.mgb_device_alloc(16, None) == mgb.INVALID_ARGUMENT


def test_embedding_arguments_are_checked_before_device_work():
    lib = mgb.lib()
    fake = 1 << 40
    # a declined format, a ragged table, null pointers
    assert lib.mgb_embedding(3, fake, 8, 256, 0, fake, 1, 0, 1.0, fake, None, None) == mgb.UNSUPPORTED
    assert lib.mgb_embedding(mgb.Q4_K, fake, 8, 96, 0, fake, 1, 0, 1.0, fake, None, None) == \
        mgb.INVALID_ARGUMENT
    assert lib.mgb_embedding(mgb.Q8_0, None, 8, 64, 0, fake, 1, 0, 1.0, fake, None, None) == \
        mgb.INVALID_ARGUMENT


@pytest.mark.parametrize("m,n,k,parts", [
    (16, 14336, 4096, 1), (16, 4096, 4096, 4), (16, 1024, 4096, 8),  # config 3, M = 16
    (512, 14336, 4096, 1), (512, 7168, 4096, 1), (512, 1792, 4096, 4),  # config 1 shards
    (2048, 8192, 8192, 1), (2048, 1024, 8192, 2), (2048, 512, 8192, 4),  # config 4, N = 1, 2
    (2048, 128, 8192, 8), (2048, 1024, 28672, 2), (65536, 64, 4096, 1)])
def test_split_choices(m, n, k, parts):
    """The K split the preferred workspace provides for the benchmark shapes and
    their tensor-parallel shards (host logic: no device work)."""
    extra = mgb.qmatmul_workspace_bytes(mgb.Q4_K, m, n, k) - \
        mgb.qmatmul_min_workspace_bytes(mgb.Q4_K, m, n, k)
    assert extra == (0 if parts == 1 else parts * m * n * 4)
