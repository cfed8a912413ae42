"""Seeded synthetic workloads with the shapes and value distributions of the
benchmark configurations (the reference has no Q4_K quantiser, so packed
weights are random bytes with controlled scale fields):

- Q4_K:   uniform bytes (uniform 4-bit quants, uniform 6-bit scales/mins),
          f16 d and dmin ~ U(1e-3, 1e-2) over bytes 0..3 of each 144-byte block;
- Q8_0:   f16 d ~ U(1e-3, 1e-2), int8 quants ~ U[-127, 127];
- IQ4_NL, Q4_0: f16 d ~ U(1e-3, 1e-2), uniform 4-bit indices;
- Q5_K:   as Q4_K over 176-byte blocks (uniform fifth bits);
- Q6_K:   uniform bytes (uniform 6-bit quants, uniform int8 scales), f16 d
          ~ U(1e-3, 1e-2) at bytes 208..209 of each 210-byte block;
- activations f32 ~ N(0, 1).
Bytes are in the ggml block layout a checkpoint holds (stored rows = output
columns).
"""

from __future__ import annotations

import numpy as np

Q8_0, Q4_K, Q6_K, IQ4_NL, Q5_K, Q4_0 = 0, 1, 2, 5, 12, 13
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210), IQ4_NL: (32, 18),
         Q4_0: (32, 18)}
SEED = 0x5EED


def _f16_field(rng: np.random.Generator, count: int) -> np.ndarray:
    return rng.uniform(1e-3, 1e-2, size=count).astype(np.float16).view(np.uint8).reshape(count, 2)


def packed_weights(fmt: int, rows: int, cols: int, seed: int = SEED) -> np.ndarray:
    elems, bb = BLOCK[fmt]
    if cols % elems:
        raise ValueError(f"cols {cols} is not a multiple of {elems}")
    rng = np.random.default_rng(seed)
    blocks = rows * cols // elems
    data = rng.integers(0, 256, size=(blocks, bb), dtype=np.uint8)
    if fmt in (Q4_K, Q5_K):
        data[:, 0:2] = _f16_field(rng, blocks)
        data[:, 2:4] = _f16_field(rng, blocks)
    elif fmt == Q6_K:
        data[:, 208:210] = _f16_field(rng, blocks)
    elif fmt == Q8_0:
        data[:, 0:2] = _f16_field(rng, blocks)
        data[:, 2:] = rng.integers(-127, 128, size=(blocks, 32), dtype=np.int8).view(np.uint8)
    else:
        data[:, 0:2] = _f16_field(rng, blocks)
    return data.reshape(-1)


def activations(m: int, k: int, seed: int = SEED + 1) -> np.ndarray:
    return np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)


def packed_nbytes(fmt: int, rows: int, cols: int) -> int:
    elems, bb = BLOCK[fmt]
    return rows * cols // elems * bb


def row_slice(fmt: int, data: np.ndarray, cols: int, rows: np.ndarray) -> np.ndarray:
    """The ggml bytes of the selected stored rows (rows are contiguous)."""
    rb = packed_nbytes(fmt, 1, cols)
    return np.ascontiguousarray(data.reshape(-1, rb)[rows]).reshape(-1)
