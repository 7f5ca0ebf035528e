#!/usr/bin/env python3
"""Generate the committed golden fixtures under tests/golden/.

Run from the repository root:  python tests/golden/make_golden.py

Fixture formats are the reference's own (tools/test_quants.c:1-13 in
rinaldofesta/sepia):
  SQFX  magic 0x58465153, <6I header (magic, ver=1, type, n_blocks,
        block_elems, block_bytes), raw blocks, then fp32 expected values.
  SQLX  magic 0x584C5153, <5I header (magic, ver=1, type, out, in), raw
        weight rows, fp32 x[in], fp32 y[out].

Expected values come from gguf-py 0.19.0's numpy `dequantize` (the library
the reference's tools/make_quant_fixtures.py uses), never from this
repository's code. Blocks are uniform random bytes with the fp16 scale
fields overwritten by finite halves (normal, subnormal and signed), the
reference generator's recipe (tools/make_quant_fixtures.py:23-32, 71-80)
widened to the four formats the reference lacks (Q2_K, Q3_K, IQ2_XXS, IQ1_S).
SQLX expectations are the double-accumulated qlinear of src/sepia.c:748-753
computed with numpy float64 over the gguf-py dequantized rows.
"""
import struct
from pathlib import Path

import numpy as np
from gguf.constants import GGML_QUANT_SIZES, GGMLQuantizationType as T
from gguf.quants import dequantize

OUT = Path(__file__).resolve().parent
SEED = 20261201
SQFX, SQLX = 0x58465153, 0x584C5153

# ggml type -> byte offsets of the fp16 scale fields inside one block
F16_FIELDS = {
    T.Q8_0: (0,), T.Q2_K: (80, 82), T.Q3_K: (108,), T.Q4_K: (0, 2), T.Q5_K: (0, 2),
    T.Q6_K: (208,), T.IQ2_XXS: (0,), T.IQ2_XS: (0,), T.IQ3_XXS: (0,), T.IQ1_S: (0,),
    T.IQ4_XS: (0,),
}


def f16_fields(rng, n):
    """Finite halves: mostly positive normals (the reference recipe), plus
    negative values, subnormals and zero so the software conversion is hit."""
    exp = rng.integers(0x01, 0x1F, size=n, dtype=np.uint16)
    mant = rng.integers(0, 0x400, size=n, dtype=np.uint16)
    bits = (exp << np.uint16(10)) | mant
    k = rng.random(n)
    bits = np.where(k < 0.15, bits | np.uint16(0x8000), bits)                 # negative
    sub = rng.integers(0, 0x400, size=n, dtype=np.uint16)
    bits = np.where((k >= 0.15) & (k < 0.25), sub, bits)                        # subnormal/zero
    return bits.astype(np.uint16)


def rand_blocks(rng, qt, nb):
    blk, tsz = GGML_QUANT_SIZES[qt]
    raw = rng.integers(0, 256, size=(nb, tsz), dtype=np.uint8)
    for off in F16_FIELDS[qt]:
        raw[:, off:off + 2] = f16_fields(rng, nb).view(np.uint8).reshape(nb, 2)
    return raw


def write_sqfx(qt, raw):
    blk, tsz = GGML_QUANT_SIZES[qt]
    nb = raw.shape[0]
    exp = dequantize(raw.reshape(-1), qt).astype(np.float32).reshape(-1)
    assert exp.size == nb * blk and np.isfinite(exp).all()
    path = OUT / f"sqfx_{qt.name.lower()}.bin"
    with open(path, "wb") as f:
        f.write(struct.pack("<6I", SQFX, 1, int(qt), nb, blk, tsz))
        f.write(raw.tobytes())
        f.write(exp.astype("<f4").tobytes())
    return path


def write_sqlx(rng, qt, out_dim, in_dim):
    blk, tsz = GGML_QUANT_SIZES[qt]
    nb_row = in_dim // blk
    raw = rand_blocks(rng, qt, out_dim * nb_row)
    w = dequantize(raw.reshape(-1), qt).astype(np.float32).reshape(out_dim, in_dim)
    x = rng.standard_normal(in_dim).astype(np.float32)
    # sequential double accumulation, as dotf does (np.cumsum is sequential)
    y = np.cumsum(w.astype(np.float64) * x.astype(np.float64), axis=1)[:, -1].astype(np.float32)
    path = OUT / f"sqlx_{qt.name.lower()}.bin"
    with open(path, "wb") as f:
        f.write(struct.pack("<5I", SQLX, 1, int(qt), out_dim, in_dim))
        f.write(raw.tobytes())
        f.write(x.astype("<f4").tobytes())
        f.write(y.astype("<f4").tobytes())
    return path


def main():
    rng = np.random.default_rng(SEED)
    # F16: every bit pattern class (zero, -0, subnormals, normals, max)
    bits = np.concatenate([np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x83FF, 0x3C00, 0xBC00, 0x7BFF, 0xFBFF],
                                    dtype=np.uint16), rng.integers(0, 0x7C00, size=55, dtype=np.uint16)])
    path = OUT / "sqfx_f16.bin"
    with open(path, "wb") as f:
        f.write(struct.pack("<6I", SQFX, 1, int(T.F16), bits.size, 1, 2))
        f.write(bits.astype("<u2").tobytes())
        f.write(bits.view(np.float16).astype(np.float32).astype("<f4").tobytes())
    print(path)
    for qt in F16_FIELDS:
        blk, _ = GGML_QUANT_SIZES[qt]
        nb = 64 if blk == 32 else 12
        print(write_sqfx(qt, rand_blocks(rng, qt, nb)))
        in_dim = 512 if blk == 256 else 128
        print(write_sqlx(rng, qt, 4, in_dim))


if __name__ == "__main__":
    main()
