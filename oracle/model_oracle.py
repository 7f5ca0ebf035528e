"""Full-model CPU restatement -- TEST INFRASTRUCTURE ONLY.

Composes the oracle's C kernels (oracle/liboracle.so) into the reference's
decoder, step for step:
  attn_chunk       attn_forward_chunk      src/sepia.c:1077-1276
  dense_mlp        mlp_dense_forward       src/sepia.c:1278-1315
  moe_mlp          mlp_moe_forward         src/sepia.c:1377-1470 (real experts:
                                           real_expert_ffn src/sepia.c:2993-3022)
  decoder_layer    decoder_layer_forward   src/sepia.c:1483-1552
  forward_chunk    real_forward_chunk      src/sepia.c:3345-3390
  generate_ids     real_generate's loop    src/sepia.c:4114-4158 (token ids in,
                                           no tokenizer)
Every float operation keeps the reference's order and precision (fp32
storage, double accumulation), so on the same container it reproduces the
reference bit for bit (tests/test_model_cpu.py checks that against the
reference compiled in place). Only tests/, smoke() and bench.py's CPU
baseline use it; nothing under sepia_b200/ imports it.
"""
from __future__ import annotations

import math

import numpy as np

from . import oracle as O


def tau_of(cfg, is_sliding: bool, q_pos: int) -> float:
    """src/sepia.c:1188-1194 (double)."""
    if is_sliding or not cfg["has_log_scaling"]:
        return 1.0
    ratio = float(q_pos + 1) / float(cfg["log_scaling_n_floor"])
    if ratio < 1.0:
        ratio = 1.0
    return 1.0 + cfg["log_scaling_alpha"] * math.log(ratio)


def attn_chunk(cfg, lw, lc, x_normed, T, start_pos, nthreads=1):
    """One attention block on fp32 weights. cfg: hidden, d_rel, conv_k,
    eps, window, has_log_scaling, log_scaling_alpha, log_scaling_n_floor;
    lw: is_sliding, H, Hkv, Dh, rel_extent, wq/wk/wv/wr/wo ([out,in] f32),
    q_norm, k_norm, rel_proj, k_sconv, v_sconv; lc: k, v ([cap, kv_dim]),
    k_hist, v_hist ([K-1, kv_dim], updated in place)."""
    hidden, K, d_rel = cfg["hidden"], cfg["conv_k"], cfg["d_rel"]
    H, Hkv, Dh, E = lw["H"], lw["Hkv"], lw["Dh"], lw["rel_extent"]
    q_dim, kv_dim = H * Dh, Hkv * Dh
    eps = np.float32(cfg["eps"])
    x_normed = np.ascontiguousarray(x_normed, np.float32).reshape(T, hidden)
    q_raw = np.stack([O.linear(lw["wq"], x_normed[t], nthreads) for t in range(T)])
    k_raw = np.stack([O.linear(lw["wk"], x_normed[t], nthreads) for t in range(T)])
    v_raw = np.stack([O.linear(lw["wv"], x_normed[t], nthreads) for t in range(T)])
    r_raw = np.stack([O.linear(lw["wr"], x_normed[t], nthreads) for t in range(T)])
    k_s = O.sconv_apply(lw["k_sconv"], kv_dim, K, lc["k_hist"], k_raw, T).reshape(T, kv_dim)
    v_s = O.sconv_apply(lw["v_sconv"], kv_dim, K, lc["v_hist"], v_raw, T).reshape(T, kv_dim)
    for t in range(T):
        for h in range(H):
            q_raw[t, h * Dh:(h + 1) * Dh] = O.rmsnorm(q_raw[t, h * Dh:(h + 1) * Dh], lw["q_norm"], eps)
        for h in range(Hkv):
            k_s[t, h * Dh:(h + 1) * Dh] = O.rmsnorm(k_s[t, h * Dh:(h + 1) * Dh], lw["k_norm"], eps)
    lc["k"][start_pos:start_pos + T] = k_s
    lc["v"][start_pos:start_pos + T] = v_s
    pos = start_pos + np.arange(T)
    tau = np.array([tau_of(cfg, lw["is_sliding"], int(p)) for p in pos], np.float64)
    if lw["is_sliding"]:
        lo = np.maximum(0, pos - cfg["window"] + 1).astype(np.int64)
    else:
        lo = np.zeros(T, np.int64)
    hi = pos.astype(np.int64)
    rl = O.rel_project(r_raw, lw["rel_proj"], T, H, d_rel, E)
    # q_scaled = (float)((double)q * tau)  (src/sepia.c:1209)
    q_scaled = (q_raw.astype(np.float64) * tau[:, None]).astype(np.float32)
    att = O.banded_attn64(q_scaled, lc["k"], lc["v"], rl, lo, hi, tau, T, H, Hkv, Dh, E, start_pos, kv_dim,
                          np.float32(1.0 / Dh), nthreads=nthreads).reshape(T, q_dim)
    return np.stack([O.linear(lw["wo"], att[t], nthreads) for t in range(T)])
