"""GPU parity of the packed-table `embedding` Kernel against the CPU oracle.

`NativeState::embedding` (src/native/mod.rs:389-417) returns, for every token
id, the dequantised row of an untransposed [vocab, dim] table or the token's
value in every stored row of a transposed [dim, vocab] one, then multiplies by
the optional `scale` attribute (:439-447).  The values are the dequantised
elements (bit-exact to `dequantize_row` / `element`), so the comparison is
bit for bit; an invalid id fails the Kernel with the reference's message.
"""

from __future__ import annotations

import numpy as np
import pytest

import magnetar_b200 as mgb

pytestmark = pytest.mark.gpu

FORMATS = [mgb.Q4_K, mgb.Q5_K, mgb.Q6_K, mgb.Q8_0, mgb.IQ4_NL, mgb.Q4_0]


@pytest.fixture(scope="module")
def torch_cuda(cuda_device):
    import torch

    torch.cuda.set_device(cuda_device)
    return torch


@pytest.fixture()
def provider(cuda_device):
    with mgb.B200Provider() as p:
        p.initialize()
        yield p


def _device_layout(torch, fmt, ggml, rows, cols):
    src = torch.from_numpy(np.ascontiguousarray(ggml)).cuda()
    out = torch.empty(mgb.packed_bytes(fmt, rows, cols), dtype=torch.uint8, device="cuda")
    mgb.repack(fmt, src.data_ptr(), rows, cols, out.data_ptr(),
               torch.cuda.current_stream().cuda_stream)
    return out


def _same_bits(a, b) -> bool:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("transposed", [False, True])
@pytest.mark.parametrize("scale", [None, 0.125, -3.0])
def test_lookup_equals_dequantised_rows(torch_cuda, oracle, fmt, transposed, scale):
    torch = torch_cuda
    # stored [rows, cols]; logical [vocab, dim]
    rows, cols = (256, 512) if transposed else (512, 256)
    w = oracle.test_packed(fmt, rows, cols, 31)
    stored = oracle.dequantize(fmt, w, rows, cols).reshape(rows, cols)
    table = stored.T if transposed else stored  # [vocab, dim]
    vocab, dim = table.shape
    ids = np.array([7, 0, vocab - 1, 7, 123, 1], dtype=np.float32)
    wdev = _device_layout(torch, fmt, w, rows, cols)
    idd = torch.from_numpy(ids).cuda()
    out = torch.full((ids.size, dim), float("nan"), dtype=torch.float32, device="cuda")
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    mgb.embedding(fmt, wdev.data_ptr(), rows, cols, transposed, idd.data_ptr(), ids.size,
                  out.data_ptr(), scale=scale, bad_ptr=bad.data_ptr(),
                  stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    expected = table[ids.astype(np.int64)]
    if scale is not None:
        expected = expected * np.float32(scale)
    assert _same_bits(out.cpu().numpy(), expected)
    assert int(bad.cpu().numpy()[0]) & 0xFFFFFFFF == 0xFFFFFFFF


def test_invalid_ids_are_located_and_zeroed(torch_cuda, oracle):
    torch = torch_cuda
    w = oracle.test_packed(mgb.Q8_0, 50, 64, 31)
    wdev = _device_layout(torch, mgb.Q8_0, w, 50, 64)
    ids = np.array([3, 49, 50, -1, 2.5, np.nan], dtype=np.float32)
    idd = torch.from_numpy(ids).cuda()
    out = torch.full((ids.size, 64), 7.0, dtype=torch.float32, device="cuda")
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    mgb.embedding(mgb.Q8_0, wdev.data_ptr(), 50, 64, False, idd.data_ptr(), ids.size,
                  out.data_ptr(), bad_ptr=bad.data_ptr(),
                  stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(bad.cpu().numpy()[0]) & 0xFFFFFFFF == 2  # the first invalid id
    got = out.cpu().numpy()
    dense = oracle.dequantize(mgb.Q8_0, w, 50, 64).reshape(50, 64)
    assert _same_bits(got[:2], dense[[3, 49]])
    assert not got[2:].any()


def test_provider_serves_packed_and_f32_tables(provider, oracle):
    # src/native/tests.rs:176-192: a Q8_0 [50, 64] untransposed table
    table = oracle.test_packed(mgb.Q8_0, 50, 64, 31)
    dense = oracle.dequantize(mgb.Q8_0, table, 50, 64).reshape(50, 64)
    assert provider.write_packed_weight_tensor("t", mgb.Q8_0, 50, 64, False, table) == "Stored"
    materialised = provider.materializations()
    got = provider.embedding(np.array([7.0]), "t")
    assert _same_bits(got, dense[[7]])
    ids = np.array([[1, 2, 3], [49, 0, 7]], dtype=np.float32)
    got = provider.embedding(ids, "t", scale=0.5)
    assert _same_bits(got, dense[ids.reshape(-1).astype(np.int64)] * np.float32(0.5))
    assert provider.materializations() == materialised  # read in place, never expanded
    # an f32 table is gathered (`f32_embedding`, src/native/mod.rs:238-263)
    provider.write_tensor("f", dense)
    assert _same_bits(provider.embedding(np.array([4.0, 9.0]), "f", scale=2.0),
                      dense[[4, 9]] * np.float32(2.0))
    # a transposed Q4_K table: stored [dim, vocab]
    w = oracle.test_packed(mgb.Q4_K, 64, 512, 5)
    stored = oracle.dequantize(mgb.Q4_K, w, 64, 512).reshape(64, 512)
    provider.write_packed_weight_tensor("tt", mgb.Q4_K, 64, 512, True, w)
    assert _same_bits(provider.embedding(np.array([0.0, 511.0, 300.0]), "tt"),
                      stored.T[[0, 511, 300]])


@pytest.mark.parametrize("raw,shown", [(-1.0, "-1"), (2.5, "2.5"), (50.0, "50"),
                                       (float("nan"), "NaN"), (1e9, "1000000000")])
def test_invalid_token_fails_with_the_reference_message(provider, oracle, raw, shown):
    table = oracle.test_packed(mgb.Q8_0, 50, 64, 31)
    provider.write_packed_weight_tensor("t", mgb.Q8_0, 50, 64, False, table)
    with pytest.raises(mgb.MgbError) as info:
        provider.embedding(np.array([1.0, raw, -7.0]), "t")
    assert info.value.status == mgb.EXECUTION_FAILED
    assert str(info.value).endswith(f"token id {shown} is not below the vocabulary size 50")
    provider.write_tensor("f", np.zeros((50, 4), np.float32))
    with pytest.raises(mgb.MgbError) as info:
        provider.embedding(np.array([raw]), "f")
    assert str(info.value).endswith(f"token id {shown} is not below the vocabulary size 50")
