"""Seeded synthetic weights in the reference's block formats.

The reference publishes no weights for its benchmark shapes, so BASELINE's
configurations are filled synthetically with the distributions they state:
quant bytes uniform random (so scale/min nibbles, grid indices and sign bits
are uniform), the fp16 scale fields (d, dmin) uniform in [1e-3, 4e-3], f32
router weights N(0, 0.02), selection bias U(-0.1, 0.1), hidden states N(0,1).

Host (numpy) generators feed the CPU oracle and the tests; the device
(torch) generators fill the multi-GB expert store for the benchmark on the
GPU, where generating it on the host would dominate the run.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from . import quants as Q

D_LO, D_HI = 1e-3, 4e-3


# ------------------------------------------------------------------ host
def blocks_host(rng: np.random.Generator, t: int, n_blocks: int, d_lo=D_LO, d_hi=D_HI) -> np.ndarray:
    """n_blocks blocks of type t as a flat uint8 array."""
    e, b = Q.BLOCK[t]
    if t == Q.F32:
        return (rng.standard_normal(n_blocks, dtype=np.float32) * 0.02).view(np.uint8).copy()
    if t == Q.F16:
        return (rng.standard_normal(n_blocks).astype(np.float16) * np.float16(0.02)).view(np.uint8).copy()
    raw = rng.integers(0, 256, size=(n_blocks, b), dtype=np.uint8)
    for off in Q.F16_FIELDS[t]:
        d = rng.uniform(d_lo, d_hi, size=n_blocks).astype(np.float16)
        raw[:, off:off + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return raw.reshape(-1)


def matrix_host(rng, t: int, out_dim: int, in_dim: int) -> np.ndarray:
    e, _ = Q.BLOCK[t]
    return blocks_host(rng, t, out_dim * (in_dim // e))


# ------------------------------------------------------------------ device
def blocks_device(gen, t: int, n_blocks: int, device="cuda", d_lo=D_LO, d_hi=D_HI):
    """Same distribution as blocks_host, generated on the GPU (torch)."""
    import torch
    e, b = Q.BLOCK[t]
    if t == Q.F32:
        return (torch.randn(n_blocks, generator=gen, device=device) * 0.02).view(torch.uint8)
    if t == Q.F16:
        return (torch.randn(n_blocks, generator=gen, device=device) * 0.02).half().view(torch.uint8)
    raw = torch.randint(0, 256, (n_blocks, b), generator=gen, device=device, dtype=torch.uint8)
    for off in Q.F16_FIELDS[t]:
        d = (torch.rand(n_blocks, generator=gen, device=device) * (d_hi - d_lo) + d_lo).half()
        raw[:, off:off + 2] = d.view(torch.uint8).view(n_blocks, 2)
    return raw.view(-1)


# ------------------------------------------------------------------ MoE layer
@dataclass
class MoeShape:
    """one MoE layer of the Inkling shape."""
    hidden: int = 7168
    ff: int = 2048
    n_routed: int = 256
    n_shared: int = 2
    topk: int = 6
    route_scale: float = 8.0
    global_scale: float = 1.0
    gate_type: int = Q.Q2_K
    up_type: int = Q.Q2_K
    down_type: int = Q.Q3_K
    sh_gate_type: int = Q.Q4_K
    sh_up_type: int = Q.Q4_K
    sh_down_type: int = Q.Q4_K

    def strides(self):
        def pad(n):  # keep every expert matrix 256-byte aligned in the store
            return (n + 255) // 256 * 256
        return (pad(Q.row_bytes(self.gate_type, self.hidden) * self.ff),
                pad(Q.row_bytes(self.up_type, self.hidden) * self.ff),
                pad(Q.row_bytes(self.down_type, self.ff) * self.hidden),
                pad(Q.row_bytes(self.sh_gate_type, self.hidden) * self.ff),
                pad(Q.row_bytes(self.sh_up_type, self.hidden) * self.ff),
                pad(Q.row_bytes(self.sh_down_type, self.ff) * self.hidden))

    def expert_bytes(self) -> int:
        return (Q.row_bytes(self.gate_type, self.hidden) * self.ff + Q.row_bytes(self.up_type, self.hidden) * self.ff
                + Q.row_bytes(self.down_type, self.ff) * self.hidden)

    def shared_bytes(self) -> int:
        return (Q.row_bytes(self.sh_gate_type, self.hidden) * self.ff
                + Q.row_bytes(self.sh_up_type, self.hidden) * self.ff
                + Q.row_bytes(self.sh_down_type, self.ff) * self.hidden)

    def router_bytes(self) -> int:
        return (self.n_routed + self.n_shared) * self.hidden * 4

    def token_bytes(self) -> int:
        """Algorithmic HBM bytes of one token through the layer: router +
        topk routed experts + shared experts + activations (x read by the
        router and the gate/up pass, h written and read, out written)."""
        acts = 4 * (2 * self.hidden + 2 * (self.topk + self.n_shared) * self.ff + self.hidden)
        return (self.router_bytes() + self.n_routed * 4 + self.topk * self.expert_bytes()
                + self.n_shared * self.shared_bytes() + acts)


@dataclass
class MoeLayerHost:
    """Numpy copy of one layer (the oracle's input layout)."""
    shape: MoeShape
    router_w: np.ndarray
    router_bias: np.ndarray
    gate: np.ndarray
    up: np.ndarray
    down: np.ndarray
    sh_gate: np.ndarray
    sh_up: np.ndarray
    sh_down: np.ndarray
    gate_stride: int = 0
    up_stride: int = 0
    down_stride: int = 0
    sh_gate_stride: int = 0
    sh_up_stride: int = 0
    sh_down_stride: int = 0
    extra: dict = field(default_factory=dict)

    def __getattr__(self, k):  # shape fields (hidden, ff, types, ...) read through
        if k != "shape" and "shape" in self.__dict__ and hasattr(self.__dict__["shape"], k):
            return getattr(self.__dict__["shape"], k)
        raise AttributeError(k)


def _store(rng, t, rows, cols, n, stride):
    out = np.zeros(n * stride, np.uint8)
    nb = Q.row_bytes(t, cols) * rows
    for e in range(n):
        out[e * stride:e * stride + nb] = matrix_host(rng, t, rows, cols)
    return out


def moe_layer_host(shape: MoeShape, seed: int = 2) -> MoeLayerHost:
    rng = np.random.default_rng(seed)
    sg, su, sd, ssg, ssu, ssd = shape.strides()
    n_total = shape.n_routed + shape.n_shared
    router_w = (rng.standard_normal((n_total, shape.hidden), dtype=np.float32) * np.float32(0.02))
    router_bias = rng.uniform(-0.1, 0.1, size=shape.n_routed).astype(np.float32)
    L = MoeLayerHost(
        shape=shape, router_w=np.ascontiguousarray(router_w), router_bias=router_bias,
        gate=_store(rng, shape.gate_type, shape.ff, shape.hidden, shape.n_routed, sg),
        up=_store(rng, shape.up_type, shape.ff, shape.hidden, shape.n_routed, su),
        down=_store(rng, shape.down_type, shape.hidden, shape.ff, shape.n_routed, sd),
        sh_gate=_store(rng, shape.sh_gate_type, shape.ff, shape.hidden, shape.n_shared, ssg),
        sh_up=_store(rng, shape.sh_up_type, shape.ff, shape.hidden, shape.n_shared, ssu),
        sh_down=_store(rng, shape.sh_down_type, shape.hidden, shape.ff, shape.n_shared, ssd),
        gate_stride=sg, up_stride=su, down_stride=sd, sh_gate_stride=ssg, sh_up_stride=ssu, sh_down_stride=ssd)
    return L


def hidden_state(seed: int, hidden: int) -> np.ndarray:
    """Hidden state for token `seed` (BASELINE: N(0,1), seeds 1-64)."""
    return np.random.default_rng(seed).standard_normal(hidden).astype(np.float32)
