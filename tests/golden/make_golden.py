"""Generate the golden dequantisation fixtures that pin the CPU oracle.

The reference's dequantisation lives in the absent crate
`magnetar-provider-api` 1.0.0 (ggml block formats; call sites
src/native/quant.rs:13-16, :100-280).  gguf-py 0.19.0 (MIT, the ggml
project's own Python implementation of the same formats) is importable in
the build container, so this script uses it as the independent definition:

- Q8_0   gguf/quants.py:378-401   value = d * q
- Q4_K   gguf/quants.py:475-523   value = (d * sc) * q - (dmin * m)
- IQ4_NL gguf/quants.py:1330-1349 value = d * kvalues[i]
- Q4_0   gguf/quants.py:220-251   value = d * (q - 8)
- Q5_K   gguf/quants.py:525-549   value = (d * sc) * q - (dmin * m), q 5-bit
- Q6_K   gguf/quants.py:552-573   value = (d * sc) * (q - 32), q 6-bit, int8 sc per 16

Each fixture holds packed bytes and gguf-py's f32 output.  Two byte sources
per format: the reference's own test generator (src/native/tests.rs:34-67,
xorshift32 with small positive f16 scales) and fully random bytes, whose
f16 fields cover zero, subnormal, normal, infinite and NaN encodings.

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent

# name, reference format code (src/native/quant.rs:71-87), block elements, block bytes
FORMATS = [("q8_0", 0, 32, 34), ("q4_k", 1, 256, 144), ("iq4_nl", 5, 32, 18), ("q4_0", 13, 32, 18),
           ("q6_k", 2, 256, 210), ("q5_k", 12, 256, 176)]


def xorshift32(state: int) -> int:
    state ^= (state << 13) & 0xFFFFFFFF
    state ^= state >> 17
    state ^= (state << 5) & 0xFFFFFFFF
    return state & 0xFFFFFFFF


def reference_packed(code: int, block_bytes: int, block_elems: int, rows: int, cols: int,
                     seed: int) -> np.ndarray:
    """src/native/tests.rs:45-67 `packed`: random bytes, then each f16 field
    overwritten with exponent 3..7 and a random mantissa."""
    half_offsets = {1: [0, 2], 12: [0, 2], 2: [208]}.get(code, [0])
    s = (seed * 2654435761 + 1) & 0xFFFFFFFF
    out = bytearray()
    for _ in range(rows * cols // block_elems):
        block = bytearray()
        for _ in range(block_bytes):
            s = xorshift32(s)
            block.append(s % 256)
        for at in half_offsets:
            s = xorshift32(s)
            exponent = 3 + s % 5
            s = xorshift32(s)
            bits = (exponent << 10) | (s % 1024)
            block[at] = bits & 0xFF
            block[at + 1] = bits >> 8
        out += block
    return np.frombuffer(bytes(out), dtype=np.uint8).copy()


def gguf_dequantize(name: str, data: np.ndarray, rows: int, cols: int) -> np.ndarray:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T

    qtype = {"q8_0": T.Q8_0, "q4_k": T.Q4_K, "iq4_nl": T.IQ4_NL, "q4_0": T.Q4_0, "q6_k": T.Q6_K,
             "q5_k": T.Q5_K}[name]
    with np.errstate(all="ignore"):
        out = quants.dequantize(data.reshape(rows, -1), qtype)
    return np.asarray(out, dtype=np.float32).reshape(rows, cols)


def main() -> None:
    import importlib.metadata

    from gguf.quants import IQ4_NL

    rng = np.random.default_rng(0x5EED)
    cases = {}
    for name, code, elems, bb in FORMATS:
        rows, cols = 8, 512
        for source in ("reference_generator", "random_bytes"):
            if source == "reference_generator":
                data = reference_packed(code, bb, elems, rows, cols, seed=11)
            else:
                data = rng.integers(0, 256, size=rows * cols // elems * bb, dtype=np.uint8)
            expected = gguf_dequantize(name, data, rows, cols)
            key = f"{name}__{source}"
            cases[key + "__bytes"] = data
            cases[key + "__expected"] = expected
            cases[key + "__meta"] = np.array([code, rows, cols], dtype=np.int64)
    cases["iq4_nl_kvalues"] = np.array(IQ4_NL.kvalues, dtype=np.int8)
    cases["gguf_version"] = np.array([importlib.metadata.version("gguf")])
    np.savez_compressed(HERE / "dequant_gguf.npz", **cases)
    print("wrote", HERE / "dequant_gguf.npz", len(cases), "arrays")


if __name__ == "__main__":
    main()
