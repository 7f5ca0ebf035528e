"""ctypes binding of libsepia_cuda.so (the C ABI in include/sepia_gpu.h and
include/sepia_cuda.h).

The library is loaded from this package directory. There is no fallback:
if the shared object is missing or does not load, `load()` raises, so a GPU
run can never silently take a CPU path.
"""
from __future__ import annotations

import ctypes as C
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsepia_cuda.so"
INCLUDE = HERE.parent / "include"

_lib = None

vp = C.c_void_p
i64 = C.c_int64
i32 = C.c_int32


class SepiaMoeLayer(C.Structure):
    _fields_ = [("hidden", i64), ("ff", i64), ("n_routed", i32), ("n_shared", i32), ("topk", i32),
                ("route_scale", C.c_double), ("global_scale", C.c_float),
                ("router_w", vp), ("router_bias", vp),
                ("gate_type", i32), ("up_type", i32), ("down_type", i32),
                ("gate", vp), ("up", vp), ("down", vp),
                ("gate_stride", i64), ("up_stride", i64), ("down_stride", i64),
                ("sh_gate_type", i32), ("sh_up_type", i32), ("sh_down_type", i32),
                ("sh_gate", vp), ("sh_up", vp), ("sh_down", vp),
                ("sh_gate_stride", i64), ("sh_up_stride", i64), ("sh_down_stride", i64),
                ("rank", i32), ("world", i32), ("expert_slot", vp)]


class SepiaMoeWork(C.Structure):
    _fields_ = [("logits", vp), ("topk_idx", vp), ("weights", vp), ("h", vp), ("slots", vp), ("counter", vp), ("router_part", vp), ("sync", vp), ("htab", vp)]


class SepiaGpuMoeDesc(C.Structure):
    _fields_ = [("hidden", i64), ("ff", i64), ("n_routed", i32), ("n_shared", i32), ("topk", i32),
                ("route_scale", C.c_double), ("global_scale", C.c_float),
                ("router_w", vp), ("router_w_off", C.c_size_t), ("router_bias", vp), ("router_bias_off", C.c_size_t),
                ("gate_type", i32), ("up_type", i32), ("down_type", i32),
                ("experts", vp), ("gate_off", C.c_size_t), ("up_off", C.c_size_t), ("down_off", C.c_size_t),
                ("gate_stride", i64), ("up_stride", i64), ("down_stride", i64),
                ("sh_gate_type", i32), ("sh_up_type", i32), ("sh_down_type", i32),
                ("shared", vp), ("sh_gate_off", C.c_size_t), ("sh_up_off", C.c_size_t), ("sh_down_off", C.c_size_t),
                ("sh_gate_stride", i64), ("sh_up_stride", i64), ("sh_down_stride", i64)]


class SepiaQTensor(C.Structure):
    _fields_ = [("type", i32), ("reserved", i32), ("data", vp), ("rows", i64), ("cols", i64)]


class SepiaModelLayer(C.Structure):
    _fields_ = [("is_sliding", i32), ("is_sparse", i32), ("n_heads", i32), ("n_kv_heads", i32), ("head_dim", i32),
                ("rel_extent", i32),
                ("attn_norm", vp), ("mlp_norm", vp), ("q_norm", vp), ("k_norm", vp), ("rel_proj", vp),
                ("k_sconv", vp), ("v_sconv", vp), ("attn_sconv", vp), ("mlp_sconv", vp),
                ("wq", SepiaQTensor), ("wk", SepiaQTensor), ("wv", SepiaQTensor), ("wr", SepiaQTensor),
                ("wo", SepiaQTensor),
                ("dense_gate", SepiaQTensor), ("dense_up", SepiaQTensor), ("dense_down", SepiaQTensor),
                ("dense_gscale", C.c_float),
                ("moe", SepiaMoeLayer)]


class SepiaModelDesc(C.Structure):
    _fields_ = [("hidden", i64), ("n_layers", i32), ("vocab", i32), ("unpadded_vocab", i32), ("d_rel", i32),
                ("conv_k", i32), ("window", i32), ("max_positions", i32), ("eps", C.c_float), ("mup", C.c_float),
                ("has_log_scaling", i32), ("log_scaling_alpha", C.c_double), ("log_scaling_n_floor", i64),
                ("embed", SepiaQTensor), ("unembed", SepiaQTensor), ("embed_norm", vp), ("final_norm", vp),
                ("layers", C.POINTER(SepiaModelLayer)), ("rank", i32), ("world", i32)]


# name -> (restype, argtypes)
_PROTOS = {
    # ---- sepia_gpu.h (reference ABI) ----
    "sepia_gpu_available": (C.c_int, []),
    "sepia_gpu_init": (C.c_int, [C.c_char_p]),
    "sepia_gpu_shutdown": (None, []),
    "sepia_gpu_device_name": (C.c_char_p, []),
    "sepia_gpu_wrap_mmap": (vp, [vp, C.c_size_t]),
    "sepia_gpu_alloc": (vp, [C.c_size_t, C.c_int]),
    "sepia_gpu_free": (None, [vp]),
    "sepia_gpu_host_ptr": (vp, [vp]),
    "sepia_gpu_gpu_addr": (C.c_uint64, [vp]),
    "sepia_gpu_selftest_touch": (C.c_int, [vp, C.c_size_t]),
    "sepia_gpu_begin": (C.c_int, []),
    "sepia_gpu_flush": (C.c_int, []),
    "sepia_gpu_end": (C.c_int, []),
    "sepia_gpu_rmsnorm": (C.c_int, [vp, vp, vp, i64, i64, C.c_float]),
    "sepia_gpu_matvec": (C.c_int, [vp, vp, vp, i64, i64]),
    "sepia_gpu_silu_mul": (C.c_int, [vp, vp, vp, i64]),
    "sepia_gpu_add": (C.c_int, [vp, vp, vp, i64]),
    "sepia_gpu_softmax": (C.c_int, [vp, vp, i64, i64]),
    "sepia_gpu_sconv": (C.c_int, [vp, vp, vp, vp, i64, i64, i64]),
    "sepia_gpu_matvec_q": (C.c_int, [C.c_int, vp, C.c_size_t, vp, vp, i64, i64]),
    "sepia_gpu_dequant_rows": (C.c_int, [C.c_int, vp, C.c_size_t, vp, i64]),
    "sepia_gpu_rel_project": (C.c_int, [vp, vp, vp, i64, i64, i64, i64]),
    "sepia_gpu_banded_attn": (C.c_int, [vp, vp, vp, vp, vp, vp, vp, vp] + [i64] * 7 + [C.c_float]),
    "sepia_gpu_matvec_off": (C.c_int, [vp, C.c_size_t, vp, vp, i64, i64]),
    "sepia_gpu_rmsnorm_off": (C.c_int, [vp, C.c_size_t, vp, vp, i64, i64, C.c_float]),
    "sepia_gpu_sconv_off": (C.c_int, [vp, C.c_size_t, vp, vp, vp, i64, i64, i64]),
    "sepia_gpu_rel_project_off": (C.c_int, [vp, vp, C.c_size_t, vp, i64, i64, i64, i64]),
    "sepia_gpu_copy": (C.c_int, [vp, C.c_size_t, vp, C.c_size_t, i64]),
    "sepia_gpu_scale": (C.c_int, [C.c_float, vp, vp, i64]),
    "sepia_gpu_sconv_hist_roll": (C.c_int, [vp, vp, i64, i64, i64]),
    "sepia_gpu_moe_layer": (C.c_int, [C.POINTER(SepiaGpuMoeDesc), vp, vp, vp, vp]),
    # ---- sepia_cuda.h (raw device pointers) ----
    "sepia_cuda_last_error": (C.c_char_p, []),
    "sepia_cuda_device_error": (C.c_int, [vp]),
    "sepia_cuda_sm_count": (C.c_int, []),
    "sepia_cuda_block_elems": (C.c_int, [C.c_int]),
    "sepia_cuda_block_bytes": (C.c_int, [C.c_int]),
    "sepia_cuda_row_bytes": (i64, [C.c_int, i64]),
    "sepia_cuda_dequant": (C.c_int, [C.c_int, vp, vp, i64, vp]),
    "sepia_cuda_matvec_q": (C.c_int, [C.c_int, vp, vp, vp, i64, i64, i64, vp]),
    "sepia_cuda_matvec_f32": (C.c_int, [vp, vp, vp, i64, i64, vp]),
    "sepia_cuda_rmsnorm": (C.c_int, [vp, vp, vp, i64, i64, C.c_float, vp]),
    "sepia_cuda_silu_mul": (C.c_int, [vp, vp, vp, i64, vp]),
    "sepia_cuda_expert_swiglu": (C.c_int, [C.c_int, vp, C.c_int, vp, C.c_int, vp, i64, i64, vp, vp, vp, vp]),
    "sepia_cuda_sconv": (C.c_int, [vp, vp, vp, vp, i64, i64, i64, vp]),
    "sepia_cuda_sconv_hist_roll": (C.c_int, [vp, vp, i64, i64, i64, vp]),
    "sepia_cuda_moe_work_bytes": (C.c_size_t, [C.POINTER(SepiaMoeLayer)]),
    "sepia_cuda_moe_work_carve": (C.c_int, [C.POINTER(SepiaMoeLayer), vp, C.c_size_t, C.POINTER(SepiaMoeWork)]),
    "sepia_cuda_moe_router": (C.c_int, [C.POINTER(SepiaMoeLayer), vp, C.POINTER(SepiaMoeWork), vp]),
    "sepia_cuda_moe_experts": (C.c_int, [C.POINTER(SepiaMoeLayer), vp, C.POINTER(SepiaMoeWork), vp, C.c_int, vp]),
    "sepia_cuda_moe_gateup": (C.c_int, [C.POINTER(SepiaMoeLayer), vp, C.POINTER(SepiaMoeWork), vp]),
    "sepia_cuda_moe_down": (C.c_int, [C.POINTER(SepiaMoeLayer), C.POINTER(SepiaMoeWork), vp, C.c_int, vp]),
    "sepia_cuda_moe_combine": (C.c_int, [C.POINTER(SepiaMoeLayer), C.POINTER(SepiaMoeWork), vp, vp]),
    "sepia_cuda_moe_layer": (C.c_int, [C.POINTER(SepiaMoeLayer), vp, C.POINTER(SepiaMoeWork), vp, vp]),
    "sepia_cuda_moe_fused_eligible": (C.c_int, [C.POINTER(SepiaMoeLayer), C.POINTER(SepiaMoeWork)]),
    "sepia_cuda_moe_layer_fused": (C.c_int, [C.POINTER(SepiaMoeLayer), vp, C.POINTER(SepiaMoeWork), vp, vp]),
    "sepia_cuda_topk_select": (C.c_int, [vp, i32, i32, vp, vp]),
    "sepia_cuda_rel_project": (C.c_int, [vp, vp, vp, i64, i64, i64, i64, vp]),
    "sepia_cuda_banded_attn_ws_bytes": (C.c_size_t, [i64, i64, i64, i64, i64]),
    "sepia_cuda_banded_attn": (C.c_int, [C.c_int, vp, vp, vp, vp, vp, vp, vp, vp] + [i64] * 7 + [C.c_float, i64, vp,
                                                                                                  C.c_size_t, vp]),
    "sepia_cuda_lib_stream": (vp, []),
    "sepia_cuda_exchange_create": (C.c_int, [i32, i64, i32, i32, C.POINTER(vp)]),
    "sepia_cuda_exchange_destroy": (None, [vp]),
    "sepia_cuda_exchange_handle": (C.c_int, [vp, vp]),
    "sepia_cuda_exchange_connect": (C.c_int, [vp, vp]),
    "sepia_cuda_moe_exchange": (C.c_int, [vp, C.POINTER(SepiaMoeLayer), C.POINTER(SepiaMoeWork), vp, vp]),
    "sepia_cuda_moe_layer_sharded": (C.c_int, [vp, C.POINTER(SepiaMoeLayer), vp, C.POINTER(SepiaMoeWork), vp, vp]),
    "sepia_cuda_fill_blocks": (C.c_int, [C.c_int, vp, i64, i64, i64, C.c_uint64, i64, i64, C.c_float, C.c_float, vp]),
    # ---- sepia_model.h (whole-token decode engine) ----
    "sepia_model_create": (C.c_int, [C.POINTER(SepiaModelDesc), C.POINTER(vp)]),
    "sepia_model_destroy": (None, [vp]),
    "sepia_model_device_bytes": (C.c_size_t, [vp]),
    "sepia_model_reset": (C.c_int, [vp, vp]),
    "sepia_model_prefill": (C.c_int, [vp, vp, i32, i32, vp]),
    "sepia_model_decode": (C.c_int, [vp, i32, vp, vp]),
    "sepia_model_logits": (vp, [vp]),
    "sepia_model_copy_logits": (C.c_int, [vp, vp, vp]),
    "sepia_model_exchange_handle": (C.c_int, [vp, vp]),
    "sepia_model_connect": (C.c_int, [vp, vp]),
    "sepia_model_position": (C.c_int, [vp, vp]),
    "sepia_cuda_test_engine_timeout": (C.c_int, [C.c_int, vp, vp, vp, i64, i64, C.c_longlong, vp]),
    "sepia_cuda_banded_attn_noalloc_max_bytes": (C.c_size_t, []),
    "sepia_cuda_banded_attn_noalloc": (C.c_int, [C.c_int, vp, vp, vp, vp, vp, vp, vp, vp] + [i64] * 7
                                       + [C.c_float, i64, vp]),
}


def header_symbols() -> list[str]:
    """Every function name declared in include/*.h."""
    names = []
    for h in sorted(INCLUDE.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(sepia_(?:gpu|cuda|model)_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def load(path: str | Path | None = None):
    """Load the CUDA library (building is __graft_entry__.build()'s job)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"sepia_b200: {p} is missing -- run `python -m sepia_b200.build` (no CPU fallback exists)")
    L = C.CDLL(str(p))
    for name, (res, args) in _PROTOS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = L
    return L


def last_error() -> str:
    e = load().sepia_cuda_last_error()
    return e.decode() if e else ""


def ok(ret: int, what: str = "call") -> None:
    """Raise with the library's message when an entry point returns 0."""
    if not ret:
        raise RuntimeError(f"sepia_b200: {what} failed: {last_error()}")
