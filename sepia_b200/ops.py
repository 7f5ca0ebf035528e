"""torch-tensor wrappers of the raw-pointer entry points (include/sepia_cuda.h).

Tensors only carry device memory and the stream here; every computation is
one of the library's CUDA kernels. Each wrapper raises if the library
rejects the call.
"""
from __future__ import annotations

import torch

from . import quants as Q
from .lib import load, ok


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _p(t: torch.Tensor) -> int:
    assert t.is_cuda and t.is_contiguous(), "expected a contiguous CUDA tensor"
    return t.data_ptr()


def dequant(t: int, raw: torch.Tensor, n: int, stream=None) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=raw.device)
    ok(load().sepia_cuda_dequant(t, _p(raw), _p(out), n, _stream(stream)), "dequant")
    return out


def matvec_q(t: int, w: torch.Tensor, x: torch.Tensor, out_dim: int, in_dim: int, w_offset: int = 0,
             stream=None) -> torch.Tensor:
    """y = W x for a quantized [out_dim, in_dim] matrix starting w_offset
    bytes into `w`. x may be [in_dim] or [n_vec, in_dim]."""
    n_vec = 1 if x.dim() == 1 else x.shape[0]
    y = torch.empty((out_dim,) if x.dim() == 1 else (n_vec, out_dim), dtype=torch.float32, device=x.device)
    ok(load().sepia_cuda_matvec_q(t, _p(w) + w_offset, _p(x), _p(y), out_dim, in_dim, n_vec, _stream(stream)),
       "matvec_q")
    return y


def matvec_f32(w: torch.Tensor, x: torch.Tensor, stream=None) -> torch.Tensor:
    y = torch.empty(w.shape[0], dtype=torch.float32, device=x.device)
    ok(load().sepia_cuda_matvec_f32(_p(w), _p(x), _p(y), w.shape[0], w.shape[1], _stream(stream)), "matvec_f32")
    return y


def topk_select(scores: torch.Tensor, k: int, stream=None) -> torch.Tensor:
    idx = torch.empty(k, dtype=torch.int32, device=scores.device)
    ok(load().sepia_cuda_topk_select(_p(scores), scores.numel(), k, _p(idx), _stream(stream)), "topk_select")
    return idx


def banded_attn(q, k, v, rel_logits, kv_lo, kv_hi, tau, T, H, Hkv, Dh, rel_extent, q_pos_base, kv_dim,
                inv_head_dim, stream=None) -> torch.Tensor:
    """k/v: fp32 or fp16 [cap, kv_dim] caches; kv_lo/kv_hi int64 and tau f32
    device tensors of length T."""
    L = load()
    kv_f16 = 1 if k.dtype == torch.float16 else 0
    max_kv = int((kv_hi - kv_lo).max().item()) + 1
    wsb = L.sepia_cuda_banded_attn_ws_bytes(T, H, Hkv, Dh, max_kv)
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=q.device)
    out = torch.empty(T * H * Dh, dtype=torch.float32, device=q.device)
    rl = _p(rel_logits) if rel_logits is not None else None
    ok(L.sepia_cuda_banded_attn(kv_f16, _p(q), _p(k), _p(v), rl, _p(out), _p(kv_lo), _p(kv_hi), _p(tau), T, H, Hkv,
                                Dh, rel_extent, q_pos_base, kv_dim, inv_head_dim, max_kv, _p(ws), wsb,
                                _stream(stream)), "banded_attn")
    return out


def rel_project(r_vec, rel_proj, T, H, d_rel, rel_extent, stream=None) -> torch.Tensor:
    out = torch.empty(T * H * rel_extent, dtype=torch.float32, device=r_vec.device)
    ok(load().sepia_cuda_rel_project(_p(r_vec), _p(rel_proj), _p(out), T, H, d_rel, rel_extent, _stream(stream)),
       "rel_project")
    return out


def device_error(stream=None) -> int:
    return load().sepia_cuda_device_error(_stream(stream))


def row_bytes(t: int, n: int) -> int:
    return Q.row_bytes(t, n)
