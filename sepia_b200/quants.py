"""ggml block geometry on the host (src/quants.c:28-56 plus ggml's Q2_K,
Q3_K, IQ2_XXS, IQ1_S) and the byte offsets of each format's fp16 scale
fields, used by the synthetic-weight generators."""
from __future__ import annotations

F32, F16, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 0, 1, 8, 10, 11, 12, 13, 14
IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S, IQ4_XS = 16, 17, 18, 19, 23

# type -> (elements per block, bytes per block)
BLOCK = {
    F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q2_K: (256, 84), Q3_K: (256, 110), Q4_K: (256, 144),
    Q5_K: (256, 176), Q6_K: (256, 210), IQ2_XXS: (256, 66), IQ2_XS: (256, 74), IQ3_XXS: (256, 98),
    IQ1_S: (256, 50), IQ4_XS: (256, 136),
}
NAMES = {F32: "f32", F16: "f16", Q8_0: "q8_0", Q2_K: "q2_k", Q3_K: "q3_k", Q4_K: "q4_k", Q5_K: "q5_k",
         Q6_K: "q6_k", IQ2_XXS: "iq2_xxs", IQ2_XS: "iq2_xs", IQ3_XXS: "iq3_xxs", IQ1_S: "iq1_s",
         IQ4_XS: "iq4_xs"}
BY_NAME = {v: k for k, v in NAMES.items()}
QUANT_TYPES = [Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, IQ2_XXS, IQ2_XS, IQ3_XXS, IQ1_S, IQ4_XS]
ALL_TYPES = [F32, F16] + QUANT_TYPES

# byte offsets of the fp16 scale fields inside one block (ggml layouts)
F16_FIELDS = {
    Q8_0: (0,), Q2_K: (80, 82), Q3_K: (108,), Q4_K: (0, 2), Q5_K: (0, 2), Q6_K: (208,),
    IQ2_XXS: (0,), IQ2_XS: (0,), IQ3_XXS: (0,), IQ1_S: (0,), IQ4_XS: (0,),
}


def block_elems(t: int) -> int:
    return BLOCK[t][0]


def block_bytes(t: int) -> int:
    return BLOCK[t][1]


def row_bytes(t: int, n: int) -> int:
    e, b = BLOCK[t]
    if n % e:
        raise ValueError(f"{NAMES[t]}: n={n} not a multiple of {e}")
    return n // e * b


def bits_per_weight(t: int) -> float:
    e, b = BLOCK[t]
    return 8.0 * b / e
