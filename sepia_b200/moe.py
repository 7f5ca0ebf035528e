"""The HBM-resident expert store and one MoE layer on the device.

Replaces the reference's SSD-streaming expert cache (src/sepia.c:2216-2470
expert store, 3052-3225 loader pool) with experts resident in HBM, sharded
by index across the GPUs of one box: routed expert e lives on rank
e % world at local slot e // world; shared expert s on rank s % world; the
f32 router is replicated. Per token every rank computes the same router and
top-k (deterministic), computes its own experts, writes each slot's term
into a [topk + n_shared, hidden] buffer (zero for slots it does not own),
and a sum all-reduce of that buffer plus an in-order combine reproduces the
single-GPU result bit for bit (x + 0 = x, and the combine order is fixed).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import quants as Q
from .lib import SepiaMoeLayer, SepiaMoeWork, load, ok
from .synth import MoeLayerHost, MoeShape, blocks_device


def owned_experts(n_routed: int, rank: int, world: int) -> list[int]:
    return [e for e in range(n_routed) if e % world == rank]


def owned_shared(n_shared: int, rank: int, world: int) -> list[int]:
    return [s for s in range(n_shared) if s % world == rank]


class Exchange:
    """The expert-sharded exchange of one rank (sepia_cuda_exchange_*): one
    kernel stores this rank's slot terms into every rank's buffers over
    NVLink and combines them; replaces the NCCL all-reduce of the slots."""

    def __init__(self, n_slots: int, hidden: int, rank: int, world: int):
        self.rank, self.world = rank, world
        h = C.c_void_p()
        ok(load().sepia_cuda_exchange_create(n_slots, hidden, rank, world, C.byref(h)), "exchange_create")
        self.h = h

    def connect(self, group=None):
        """Gathers every rank's 64-byte IPC handle over torch.distributed (a
        host object all-gather) and opens the peers' buffers."""
        import torch.distributed as dist
        mine = (C.c_char * 64)()
        ok(load().sepia_cuda_exchange_handle(self.h, mine), "exchange_handle")
        allh = [None] * self.world
        dist.all_gather_object(allh, bytes(mine), group=group)
        buf = (C.c_char * (64 * self.world)).from_buffer_copy(b"".join(allh))
        ok(load().sepia_cuda_exchange_connect(self.h, buf), "exchange_connect")

    def __del__(self):
        if getattr(self, "h", None):
            try:
                load().sepia_cuda_exchange_destroy(self.h)
            except Exception:
                pass
            self.h = None


class MoeLayerDevice:
    """One layer's weights on this GPU (this rank's shard) plus scratch."""

    def __init__(self, shape: MoeShape, router_w, router_bias, gate, up, down, sh_gate, sh_up, sh_down,
                 rank: int = 0, world: int = 1):
        self.shape = shape
        self.rank, self.world = rank, world
        self.router_w, self.router_bias = router_w, router_bias
        self.gate, self.up, self.down = gate, up, down
        self.sh_gate, self.sh_up, self.sh_down = sh_gate, sh_up, sh_down
        self.strides = shape.strides()
        self._struct = self._build_struct()
        L = load()
        nb = L.sepia_cuda_moe_work_bytes(C.byref(self._struct))
        self.ws_mem = torch.zeros(nb + 256, dtype=torch.uint8, device=router_w.device)
        base = (self.ws_mem.data_ptr() + 255) // 256 * 256
        self.ws = SepiaMoeWork()
        ok(L.sepia_cuda_moe_work_carve(C.byref(self._struct), base, nb, C.byref(self.ws)), "moe_work_carve")
        n_slots = shape.topk + shape.n_shared
        off = self.ws.slots - self.ws_mem.data_ptr()
        self.slots = self.ws_mem[off:off + n_slots * shape.hidden * 4].view(torch.float32).view(n_slots, shape.hidden)
        self.h = self._view(self.ws.h, n_slots * shape.ff, torch.float32).view(n_slots, shape.ff)
        self.topk_idx = self._view(self.ws.topk_idx, shape.topk, torch.int32)
        self.weights = self._view(self.ws.weights, n_slots, torch.float32)
        self.logits = self._view(self.ws.logits, shape.n_routed + shape.n_shared, torch.float32)

    def _view(self, ptr, n, dtype):
        off = ptr - self.ws_mem.data_ptr()
        esz = torch.tensor([], dtype=dtype).element_size()
        return self.ws_mem[off:off + n * esz].view(dtype)

    def _build_struct(self) -> SepiaMoeLayer:
        s = self.shape
        sg, su, sd, ssg, ssu, ssd = self.strides
        L = SepiaMoeLayer()
        L.hidden, L.ff = s.hidden, s.ff
        L.n_routed, L.n_shared, L.topk = s.n_routed, s.n_shared, s.topk
        L.route_scale, L.global_scale = s.route_scale, s.global_scale
        L.router_w, L.router_bias = self.router_w.data_ptr(), self.router_bias.data_ptr()
        L.gate_type, L.up_type, L.down_type = s.gate_type, s.up_type, s.down_type
        L.gate, L.up, L.down = self.gate.data_ptr(), self.up.data_ptr(), self.down.data_ptr()
        L.gate_stride, L.up_stride, L.down_stride = sg, su, sd
        L.sh_gate_type, L.sh_up_type, L.sh_down_type = s.sh_gate_type, s.sh_up_type, s.sh_down_type
        if s.n_shared:
            L.sh_gate, L.sh_up, L.sh_down = self.sh_gate.data_ptr(), self.sh_up.data_ptr(), self.sh_down.data_ptr()
        L.sh_gate_stride, L.sh_up_stride, L.sh_down_stride = ssg, ssu, ssd
        L.rank, L.world = self.rank, self.world
        L.expert_slot = None
        return L

    # -------------------------------------------------------- construction
    @classmethod
    def from_host(cls, H: MoeLayerHost, device="cuda", rank: int = 0, world: int = 1) -> "MoeLayerDevice":
        s = H.shape
        sg, su, sd, ssg, ssu, ssd = s.strides()
        mine = owned_experts(s.n_routed, rank, world)

        def shard(buf, stride, ids):
            out = np.zeros(max(1, len(ids)) * stride, np.uint8)
            for i, e in enumerate(ids):
                out[i * stride:(i + 1) * stride] = buf[e * stride:(e + 1) * stride]
            return torch.from_numpy(out).to(device)

        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
        return cls(s, dev(H.router_w), dev(H.router_bias), shard(H.gate, sg, mine), shard(H.up, su, mine),
                   shard(H.down, sd, mine), dev(H.sh_gate), dev(H.sh_up), dev(H.sh_down), rank, world)

    @classmethod
    def random(cls, shape: MoeShape, seed: int = 2, device="cuda", rank: int = 0, world: int = 1) -> "MoeLayerDevice":
        """Generated on the GPU; expert e's bytes depend only on (seed, e),
        never on the sharding, so every world size sees the same model."""
        s = shape
        sg, su, sd, ssg, ssu, ssd = s.strides()
        gen = torch.Generator(device=device)
        gen.manual_seed(seed)
        n_total = s.n_routed + s.n_shared
        router_w = torch.randn(n_total, s.hidden, generator=gen, device=device) * 0.02
        router_bias = torch.rand(s.n_routed, generator=gen, device=device) * 0.2 - 0.1
        mine = owned_experts(s.n_routed, rank, world)

        def store(t, rows, cols, stride, ids, tag):
            out = torch.zeros(max(1, len(ids)) * stride, dtype=torch.uint8, device=device)
            nb = Q.row_bytes(t, cols) * rows
            e_blocks = nb // Q.block_bytes(t)
            for i, e in enumerate(ids):
                gen.manual_seed(seed * 1000003 + tag * 4099 + e)
                out[i * stride:i * stride + nb] = blocks_device(gen, t, e_blocks, device)
            return out

        gate = store(s.gate_type, s.ff, s.hidden, sg, mine, 1)
        up = store(s.up_type, s.ff, s.hidden, su, mine, 2)
        down = store(s.down_type, s.hidden, s.ff, sd, mine, 3)
        sh = list(range(s.n_shared))
        sh_gate = store(s.sh_gate_type, s.ff, s.hidden, ssg, sh, 4)
        sh_up = store(s.sh_up_type, s.ff, s.hidden, ssu, sh, 5)
        sh_down = store(s.sh_down_type, s.hidden, s.ff, ssd, sh, 6)
        return cls(s, router_w.contiguous(), router_bias.contiguous(), gate, up, down, sh_gate, sh_up, sh_down,
                   rank, world)

    def expert_bytes_host(self, e: int):
        """Host copies of routed expert e's (gate, up, down) bytes (this rank
        must own e)."""
        assert e % self.world == self.rank
        i = e // self.world if self.world > 1 else e
        sg, su, sd = self.strides[:3]
        s = self.shape
        ng = Q.row_bytes(s.gate_type, s.hidden) * s.ff
        nu = Q.row_bytes(s.up_type, s.hidden) * s.ff
        nd = Q.row_bytes(s.down_type, s.ff) * s.hidden
        return (self.gate[i * sg:i * sg + ng].cpu().numpy(), self.up[i * su:i * su + nu].cpu().numpy(),
                self.down[i * sd:i * sd + nd].cpu().numpy())

    # -------------------------------------------------------------- compute
    @property
    def struct(self) -> SepiaMoeLayer:
        return self._struct

    def forward(self, x: torch.Tensor, out: torch.Tensor, stream=None, group=None) -> torch.Tensor:
        """out[hidden] = MoE(x[hidden]) on this rank. For world > 1 the slot
        terms are combined through self.exchange (an Exchange, set by the
        caller) when present, else all-reduced over `group` with NCCL."""
        L = load()
        st = (stream or torch.cuda.current_stream()).cuda_stream
        Ls, ws = C.byref(self._struct), C.byref(self.ws)
        if self.world == 1:
            ok(L.sepia_cuda_moe_layer(Ls, x.data_ptr(), ws, out.data_ptr(), st), "moe_layer")
            return out
        if getattr(self, "exchange", None) is not None:
            ok(L.sepia_cuda_moe_layer_sharded(self.exchange.h, Ls, x.data_ptr(), ws, out.data_ptr(), st),
               "moe_layer_sharded")
            return out
        import torch.distributed as dist
        ok(L.sepia_cuda_moe_router(Ls, x.data_ptr(), ws, st), "moe_router")
        ok(L.sepia_cuda_moe_experts(Ls, x.data_ptr(), ws, None, 1, st), "moe_experts")
        dist.all_reduce(self.slots, op=dist.ReduceOp.SUM, group=group)
        ok(L.sepia_cuda_moe_combine(Ls, ws, out.data_ptr(), st), "moe_combine")
        return out
