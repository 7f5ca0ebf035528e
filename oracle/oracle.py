"""ctypes bindings for the CPU checker -- TEST INFRASTRUCTURE ONLY.

Loads oracle/liboracle.so (the C restatement) and, when it was built,
oracle/_ref/libsepia_ref.so (the reference's own src/sepia.c + src/quants.c,
compiled in place). Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline import this module; the CUDA library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None
_REF = None

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
I64P = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
U8P = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")

T_F32, T_F16, T_Q8_0, T_Q2_K, T_Q3_K, T_Q4_K, T_Q5_K, T_Q6_K = 0, 1, 8, 10, 11, 12, 13, 14
T_IQ2_XXS, T_IQ2_XS, T_IQ3_XXS, T_IQ1_S, T_IQ4_XS = 16, 17, 18, 19, 23
ALL_TYPES = [T_F32, T_F16, T_Q8_0, T_Q2_K, T_Q3_K, T_Q4_K, T_Q5_K, T_Q6_K,
             T_IQ2_XXS, T_IQ2_XS, T_IQ3_XXS, T_IQ1_S, T_IQ4_XS]
TYPE_NAMES = {T_F32: "f32", T_F16: "f16", T_Q8_0: "q8_0", T_Q2_K: "q2_k", T_Q3_K: "q3_k",
              T_Q4_K: "q4_k", T_Q5_K: "q5_k", T_Q6_K: "q6_k", T_IQ2_XXS: "iq2_xxs",
              T_IQ2_XS: "iq2_xs", T_IQ3_XXS: "iq3_xxs", T_IQ1_S: "iq1_s", T_IQ4_XS: "iq4_xs"}
# the nine formats src/quants.c implements (src/quants.h:6-10)
REF_TYPES = [T_F32, T_F16, T_Q8_0, T_Q4_K, T_Q5_K, T_Q6_K, T_IQ2_XS, T_IQ3_XXS, T_IQ4_XS]


def build(quiet: bool = True) -> None:
    """make -C oracle (the restatement always; _ref when the reference exists)."""
    out = subprocess.run(["make", "-C", str(HERE)], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)


def lib():
    global _LIB
    if _LIB is None:
        path = HERE / "liboracle.so"
        if not path.exists():
            build()
        L = C.CDLL(str(path))
        L.or_block_size.restype = C.c_int64
        L.or_block_size.argtypes = [C.c_int]
        L.or_type_size.restype = C.c_size_t
        L.or_type_size.argtypes = [C.c_int]
        L.or_row_bytes.restype = C.c_size_t
        L.or_row_bytes.argtypes = [C.c_int, C.c_int64]
        L.or_dequantize_row.restype = C.c_int
        L.or_dequantize_row.argtypes = [C.c_int, C.c_void_p, F32P, C.c_int64]
        L.or_qlinear.restype = C.c_int
        L.or_qlinear.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, F32P, F32P, C.c_int]
        L.or_qlinear_batch.restype = C.c_int
        L.or_qlinear_batch.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, C.c_int64, F32P, F32P, C.c_int]
        L.or_linear.argtypes = [F32P, C.c_int64, C.c_int64, F32P, F32P, C.c_int]
        L.or_rmsnorm.argtypes = [F32P, F32P, C.c_int64, C.c_float, F32P]
        L.or_silu_mul.argtypes = [F32P, F32P, F32P, C.c_int64]
        L.or_softmax_rows.argtypes = [F32P, F32P, C.c_int64, C.c_int64]
        L.or_sconv_apply.argtypes = [F32P, C.c_int64, C.c_int64, F32P, F32P, C.c_int64, F32P]
        L.or_sconv_nohist.argtypes = [F32P, F32P, F32P, F32P, C.c_int64, C.c_int64, C.c_int64]
        L.or_sconv_hist_roll.argtypes = [F32P, F32P, C.c_int64, C.c_int64, C.c_int64]
        L.or_route_select.argtypes = [C.c_int, C.c_int, C.c_int, C.c_double, C.c_float,
                                      F32P, F32P, I32P, F32P]
        L.or_topk_scores.argtypes = [C.c_int, C.c_int, F32P, I32P]
        L.or_expert_swiglu.restype = C.c_int
        L.or_expert_swiglu.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                       C.c_int64, C.c_int64, C.c_float, F32P, F32P, C.c_int]
        L.or_rel_project.argtypes = [F32P, F32P, F32P, C.c_int64, C.c_int64, C.c_int64, C.c_int64]
        L.or_banded_attn.argtypes = [F32P, F32P, F32P, F32P, F32P, I64P, I64P, F32P] + \
            [C.c_int64] * 7 + [C.c_float, C.c_int]
        L.or_moe_layer.restype = C.c_int
        L.or_moe_layer.argtypes = [C.c_void_p, F32P, F32P, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.or_banded_attn64.argtypes = [F32P, F32P, F32P, F32P, F32P, I64P, I64P,
                                       np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")] + \
            [C.c_int64] * 7 + [C.c_float, C.c_int]
        L.or_f16_to_f32.restype = C.c_float
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own CPU code (None when oracle/_ref was not built)."""
    global _REF
    if _REF is None:
        path = HERE / "_ref" / "libsepia_ref.so"
        if not path.exists():
            return None
        R = C.CDLL(str(path))
        R.ref_quants_supported.restype = C.c_int
        R.ref_quants_supported.argtypes = [C.c_int]
        R.ref_dequantize_row.restype = C.c_int
        R.ref_dequantize_row.argtypes = [C.c_int, C.c_void_p, F32P, C.c_int64]
        R.ref_qlinear.restype = C.c_int
        R.ref_qlinear.argtypes = [C.c_int, C.c_void_p, C.c_int64, C.c_int64, F32P, F32P, C.c_int]
        R.ref_route_select.argtypes = [C.c_int, C.c_int, C.c_int, C.c_double, C.c_float,
                                       F32P, F32P, I32P, F32P]
        R.ref_rmsnorm.argtypes = [F32P, F32P, C.c_int, C.c_float, F32P]
        R.ref_sconv_apply.argtypes = [F32P, C.c_int, C.c_int, F32P, F32P, C.c_int, F32P]
        R.ref_attn_chunk.argtypes = [C.c_int] * 7 + [C.c_int, C.c_int, C.c_float, C.c_int, C.c_double, C.c_long] + \
            [F32P] * 14 + [F32P, C.c_int, C.c_int, F32P]
        R.ref_generate_ids.restype = C.c_int
        R.ref_generate_ids.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, I32P, C.c_int, C.c_int, I32P, C.c_void_p]
        _REF = R
    return _REF


def ref_generate(container_dir, prompt, n_gen, with_logits=True):
    """The reference's own greedy loop on a container (oracle/_ref): returns
    (ids [n_gen], logits [n_gen, unpadded] or None). None without _ref."""
    R = ref_lib()
    if R is None:
        return None
    import json
    d = Path(container_dir)
    tc = json.loads((d / "config.json").read_text())["text_config"]
    prompt = np.ascontiguousarray(prompt, np.int32)
    ids = np.zeros(n_gen, np.int32)
    logits = np.zeros((n_gen, tc["unpadded_vocab_size"]), np.float32) if with_logits else None
    R.ref_generate_ids(str(d / "config.json").encode(), str(d / "resident-manifest.json").encode(),
                       str(d / "index.json").encode(), prompt, len(prompt), n_gen, ids,
                       logits.ctypes.data if with_logits else None)
    return ids, logits


# ---------------------------------------------------------------- helpers
def block_size(t: int) -> int:
    return int(lib().or_block_size(t))


def type_size(t: int) -> int:
    return int(lib().or_type_size(t))


def row_bytes(t: int, n: int) -> int:
    return int(lib().or_row_bytes(t, n))


def _ptr(a: np.ndarray) -> int:
    assert a.flags.c_contiguous
    return a.ctypes.data


def dequantize(t: int, raw: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    if not lib().or_dequantize_row(t, _ptr(raw), out, n):
        raise ValueError(f"oracle: cannot dequantize type {t} n={n}")
    return out


def qlinear(t: int, w: np.ndarray, out_dim: int, in_dim: int, x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    y = np.empty(out_dim, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    if not lib().or_qlinear(t, _ptr(w), out_dim, in_dim, x, y, nthreads):
        raise ValueError("oracle: qlinear failed")
    return y


def qlinear_batch(t: int, w: np.ndarray, out_dim: int, in_dim: int, X: np.ndarray, nthreads: int = 1) -> np.ndarray:
    """[n_vec, in_dim] vectors through one matrix; row v equals qlinear(X[v])."""
    X = np.ascontiguousarray(X, np.float32)
    y = np.empty((X.shape[0], out_dim), np.float32)
    if not lib().or_qlinear_batch(t, _ptr(w), out_dim, in_dim, X.shape[0], X.reshape(-1), y.reshape(-1), nthreads):
        raise ValueError("oracle: qlinear_batch failed")
    return y


def linear(w: np.ndarray, x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty(w.shape[0], np.float32)
    lib().or_linear(w, w.shape[0], w.shape[1], np.ascontiguousarray(x, np.float32), y, nthreads)
    return y


def route_select(logits, bias, n_routed, n_shared, topk, route_scale, global_scale):
    idx = np.empty(topk, np.int32)
    w = np.empty(topk + n_shared, np.float32)
    lib().or_route_select(n_routed, n_shared, topk, route_scale, global_scale,
                          np.ascontiguousarray(logits, np.float32), np.ascontiguousarray(bias, np.float32), idx, w)
    return idx, w


def topk_scores(scores, topk):
    idx = np.empty(topk, np.int32)
    lib().or_topk_scores(len(scores), topk, np.ascontiguousarray(scores, np.float32), idx)
    return idx


def expert_swiglu(gt, g, ut, u, dt, d, hidden, ff, x, h_scale=1.0, nthreads=1):
    y = np.empty(hidden, np.float32)
    if not lib().or_expert_swiglu(gt, _ptr(g), ut, _ptr(u), dt, _ptr(d), hidden, ff, h_scale,
                                  np.ascontiguousarray(x, np.float32), y, nthreads):
        raise ValueError("oracle: expert_swiglu failed")
    return y


class _MoeLayer(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("ff", C.c_int64), ("n_routed", C.c_int), ("n_shared", C.c_int),
                ("topk", C.c_int), ("route_scale", C.c_double), ("global_scale", C.c_float),
                ("router_w", C.c_void_p), ("router_bias", C.c_void_p),
                ("gate_type", C.c_int), ("up_type", C.c_int), ("down_type", C.c_int),
                ("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("gate_stride", C.c_size_t), ("up_stride", C.c_size_t), ("down_stride", C.c_size_t),
                ("sh_gate_type", C.c_int), ("sh_up_type", C.c_int), ("sh_down_type", C.c_int),
                ("sh_gate", C.c_void_p), ("sh_up", C.c_void_p), ("sh_down", C.c_void_p),
                ("sh_gate_stride", C.c_size_t), ("sh_up_stride", C.c_size_t), ("sh_down_stride", C.c_size_t)]


def moe_layer(layer, x, nthreads=1):
    """layer: sepia_b200.synth.MoeLayerHost (numpy arrays). Returns
    (out, logits, topk_idx, weights)."""
    s = _MoeLayer()
    s.hidden, s.ff = layer.hidden, layer.ff
    s.n_routed, s.n_shared, s.topk = layer.n_routed, layer.n_shared, layer.topk
    s.route_scale, s.global_scale = layer.route_scale, layer.global_scale
    s.router_w, s.router_bias = _ptr(layer.router_w), _ptr(layer.router_bias)
    s.gate_type, s.up_type, s.down_type = layer.gate_type, layer.up_type, layer.down_type
    s.gate, s.up, s.down = _ptr(layer.gate), _ptr(layer.up), _ptr(layer.down)
    s.gate_stride, s.up_stride, s.down_stride = layer.gate_stride, layer.up_stride, layer.down_stride
    s.sh_gate_type, s.sh_up_type, s.sh_down_type = layer.sh_gate_type, layer.sh_up_type, layer.sh_down_type
    s.sh_gate, s.sh_up, s.sh_down = _ptr(layer.sh_gate), _ptr(layer.sh_up), _ptr(layer.sh_down)
    s.sh_gate_stride, s.sh_up_stride, s.sh_down_stride = \
        layer.sh_gate_stride, layer.sh_up_stride, layer.sh_down_stride
    n_total = layer.n_routed + layer.n_shared
    out = np.empty(layer.hidden, np.float32)
    logits = np.empty(n_total, np.float32)
    idx = np.empty(layer.topk, np.int32)
    w = np.empty(layer.topk + layer.n_shared, np.float32)
    ok = lib().or_moe_layer(C.byref(s), np.ascontiguousarray(x, np.float32), out,
                            _ptr(logits), _ptr(idx), _ptr(w), nthreads)
    if not ok:
        raise ValueError("oracle: moe_layer failed")
    return out, logits, idx, w


def rel_project(r_vec, rel_proj, T, H, d_rel, rel_extent):
    out = np.empty(T * H * rel_extent, np.float32)
    lib().or_rel_project(np.ascontiguousarray(r_vec, np.float32), np.ascontiguousarray(rel_proj, np.float32),
                         out, T, H, d_rel, rel_extent)
    return out


def banded_attn(q, k, v, rel_logits, kv_lo, kv_hi, tau, T, H, Hkv, Dh, rel_extent, q_pos_base, kv_dim,
                inv_head_dim, nthreads=1):
    out = np.empty(T * H * Dh, np.float32)
    lib().or_banded_attn(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                         np.ascontiguousarray(v, np.float32), np.ascontiguousarray(rel_logits, np.float32),
                         out, np.ascontiguousarray(kv_lo, np.int64), np.ascontiguousarray(kv_hi, np.int64),
                         np.ascontiguousarray(tau, np.float32), T, H, Hkv, Dh, rel_extent, q_pos_base, kv_dim,
                         inv_head_dim, nthreads)
    return out


def banded_attn64(q, k, v, rel_logits, kv_lo, kv_hi, tau64, T, H, Hkv, Dh, rel_extent, q_pos_base, kv_dim,
                  inv_head_dim, nthreads=1):
    """banded_attn with tau in double, as attn_forward_chunk holds it."""
    out = np.empty(T * H * Dh, np.float32)
    lib().or_banded_attn64(np.ascontiguousarray(q, np.float32), np.ascontiguousarray(k, np.float32),
                           np.ascontiguousarray(v, np.float32), np.ascontiguousarray(rel_logits, np.float32),
                           out, np.ascontiguousarray(kv_lo, np.int64), np.ascontiguousarray(kv_hi, np.int64),
                           np.ascontiguousarray(tau64, np.float64), T, H, Hkv, Dh, rel_extent, q_pos_base, kv_dim,
                           inv_head_dim, nthreads)
    return out


def rmsnorm(x, w, eps):
    """src/sepia.c:720-729 on one row."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().or_rmsnorm(x, np.ascontiguousarray(w, np.float32), x.size, np.float32(eps), out)
    return out


def sconv_apply(w, C_, K, hist, inp, T):
    """src/sepia.c:801-816; hist ([K-1, C]) is updated in place."""
    assert hist.dtype == np.float32 and hist.flags.c_contiguous
    out = np.empty(T * C_, np.float32)
    lib().or_sconv_apply(np.ascontiguousarray(w, np.float32), C_, K, hist, np.ascontiguousarray(inp, np.float32),
                         T, out)
    return out


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """Max relative error with the reference's floored denominator
    (src/sepia.c:4584-4589): |got-want| / max(|want|, max(1e-6, 1e-3*max|want|))."""
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    if want.size == 0:
        return 0.0
    scale = float(np.max(np.abs(want)))
    floor = max(1e-6, 1e-3 * scale)
    den = np.maximum(np.abs(want), floor)
    return float(np.max(np.abs(got - want) / den))


def nproc() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # pragma: no cover
        return os.cpu_count() or 1
