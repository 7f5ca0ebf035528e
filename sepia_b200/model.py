"""A whole model on the GPU: weights resident in HBM, decode through the
native engine (include/sepia_model.h, csrc/model.cu).

  DeviceModel.from_container(dir)   loads the reference's container
      (config.json, resident.bin + manifest, index + GGUF parts): resident
      tensors are copied to the device as they are (GGUF block layout, no
      repacking), each routed expert's gate/up/down slab goes straight to
      the rank that owns it (expert e -> rank e % world, local slot
      e // world). Replaces real_load + the SSD expert cache
      (src/sepia.c:2647-2860, 2216-2470).
  DeviceModel.synthetic(cfg, types, seed)   the same layout generated on the
      device (multi-GB synthetic models for the benchmark).
  generate(prompt, n_gen)           prefill + greedy decode, token ids in and
      out (real_generate's loop, src/sepia.c:4114-4158, without the
      tokenizer).
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import quants as Q
from . import synth
from .container import Container, ModelConfig, ModelTypes, resident_specs, tensor_nbytes
from .lib import SepiaModelDesc, SepiaModelLayer, SepiaMoeLayer, SepiaQTensor, load, ok


def _pad256(n: int) -> int:
    return (n + 255) // 256 * 256


class DeviceModel:
    def __init__(self, cfg: ModelConfig, max_positions: int, rank: int = 0, world: int = 1, device="cuda"):
        self.cfg = cfg
        self.max_positions = int(max_positions)
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.t = {}          # name -> (ggml_type, gguf_shape, device tensor)
        self.experts = {}    # layer -> {slot: (type, stride, device uint8 tensor of the owned slabs)}
        self._h = None

    # ------------------------------------------------------------ loading
    @classmethod
    def from_container(cls, path, max_positions: int = 1024, rank: int = 0, world: int = 1, device="cuda"):
        ct = Container(path)
        m = cls(ct.cfg, max_positions, rank, world, device)
        for name in ct.tensors:
            t, shape, buf = ct.resident(name)
            m.t[name] = (t, shape, torch.from_numpy(np.array(buf)).to(m.device))
        for l in range(ct.cfg.num_hidden_layers):
            if not ct.cfg.layer_is_sparse[l]:
                continue
            m.experts[l] = {}
            for slot in ("gate", "up", "down"):
                t, nb, _ = ct.expert_layer(l, slot)
                stride = _pad256(nb)
                mine = m.owned()
                host = np.zeros(max(1, len(mine)) * stride, np.uint8)
                for i, e in enumerate(mine):
                    host[i * stride:i * stride + nb] = np.frombuffer(ct.expert_bytes(l, slot, e), np.uint8)
                m.experts[l][slot] = (t, stride, torch.from_numpy(host).to(m.device))
        ct.close()
        m._build()
        return m

    @classmethod
    def synthetic(cls, cfg: ModelConfig, types: ModelTypes | None = None, seed: int = 7, max_positions: int = 1024,
                  rank: int = 0, world: int = 1, device="cuda"):
        """Seeded random weights generated in HBM in BASELINE's
        distributions (sepia_cuda_fill_blocks for the quantized tensors).
        Every tensor and every routed expert has its own unit id, so a rank's
        shard holds the bytes those experts have on one GPU."""
        types = types or ModelTypes()
        m = cls(cfg, max_positions, rank, world, device)
        L = load()
        st = torch.cuda.current_stream(m.device).cuda_stream
        gen = torch.Generator(device=m.device)
        specs = resident_specs(cfg, types)
        for i, (name, t, shape) in enumerate(specs):
            if t == Q.F32:
                gen.manual_seed(seed * 1000003 + i)
                n = int(np.prod(shape))
                if name.endswith("norm.weight"):
                    v = 1.0 + torch.randn(n, generator=gen, device=m.device) * 0.1
                elif name.endswith("ffn_gate_inp.weight"):
                    v = torch.randn(n, generator=gen, device=m.device) * 0.02
                elif name.endswith("exp_probs_b.bias"):
                    v = torch.rand(n, generator=gen, device=m.device) * 0.2 - 0.1
                elif name.endswith("ffn_gscale.weight"):
                    v = torch.ones(n, device=m.device)
                elif name.endswith("attn_rel_proj.weight"):
                    v = torch.randn(n, generator=gen, device=m.device) * 0.02
                else:
                    v = torch.randn(n, generator=gen, device=m.device) * 0.1
                m.t[name] = (t, shape, v.float().contiguous().view(torch.uint8))
            else:
                nbytes = tensor_nbytes(t, shape)
                buf = torch.empty(nbytes, dtype=torch.uint8, device=m.device)
                ok(L.sepia_cuda_fill_blocks(t, buf.data_ptr(), 1, nbytes, nbytes // Q.block_bytes(t), seed, i, 1,
                                            synth.D_LO, synth.D_HI, st), "fill_blocks")
                m.t[name] = (t, shape, buf)
        H, ff, n_e = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts
        mine = m.owned()
        for l in range(cfg.num_hidden_layers):
            if not cfg.layer_is_sparse[l]:
                continue
            m.experts[l] = {}
            for k, (slot, t, rows, cols) in enumerate([("gate", types.gate, ff, H), ("up", types.up, ff, H),
                                                        ("down", types.down, H, ff)]):
                nb = Q.row_bytes(t, cols) * rows
                stride = _pad256(nb)
                buf = torch.zeros(max(1, len(mine)) * stride, dtype=torch.uint8, device=m.device)
                if mine:
                    base = (1 << 40) + (l * 3 + k) * n_e
                    ok(L.sepia_cuda_fill_blocks(t, buf.data_ptr(), len(mine), stride, nb // Q.block_bytes(t), seed,
                                                base + rank, world, synth.D_LO, synth.D_HI, st), "fill_blocks")
                m.experts[l][slot] = (t, stride, buf)
        torch.cuda.synchronize(m.device)
        m._build()
        return m

    def owned(self) -> list[int]:
        return [e for e in range(self.cfg.n_routed_experts) if e % self.world == self.rank]

    def weight_bytes(self) -> int:
        n = sum(v[2].numel() for v in self.t.values())
        for d in self.experts.values():
            n += sum(v[2].numel() for v in d.values())
        return n

    # ----------------------------------------------------------- native
    def _q(self, name, rows=None, cols=None) -> SepiaQTensor:
        t, shape, buf = self.t[name]
        q = SepiaQTensor()
        q.type = t
        q.data = buf.data_ptr()
        q.cols = shape[0]
        q.rows = int(np.prod(shape[1:]))
        return q

    def _f(self, name) -> int:
        return self.t[name][2].data_ptr()

    def _host_f32(self, name) -> np.ndarray:
        return self.t[name][2].view(torch.float32).cpu().numpy()

    def _build(self):
        cfg = self.cfg
        L = load()
        n = cfg.num_hidden_layers
        self._layers = (SepiaModelLayer * n)()
        for l in range(n):
            b = f"blk.{l}."
            Ly = self._layers[l]
            nh, nkv, dh = cfg.heads(l)
            Ly.is_sliding = int(cfg.layer_is_sliding[l])
            Ly.is_sparse = int(cfg.layer_is_sparse[l])
            Ly.n_heads, Ly.n_kv_heads, Ly.head_dim = nh, nkv, dh
            Ly.rel_extent = cfg.layer_rel_extent(l)
            Ly.attn_norm, Ly.mlp_norm = self._f(b + "attn_norm.weight"), self._f(b + "ffn_norm.weight")
            Ly.q_norm, Ly.k_norm = self._f(b + "attn_q_norm.weight"), self._f(b + "attn_k_norm.weight")
            Ly.rel_proj = self._f(b + "attn_rel_proj.weight")
            Ly.k_sconv, Ly.v_sconv = self._f(b + "shortconv_k.weight"), self._f(b + "shortconv_v.weight")
            Ly.attn_sconv, Ly.mlp_sconv = self._f(b + "shortconv_attn.weight"), self._f(b + "shortconv_mlp.weight")
            Ly.wq, Ly.wk, Ly.wv = self._q(b + "attn_q.weight"), self._q(b + "attn_k.weight"), self._q(b + "attn_v.weight")
            Ly.wr, Ly.wo = self._q(b + "attn_r.weight"), self._q(b + "attn_output.weight")
            gscale = float(self._host_f32(b + "ffn_gscale.weight")[0])
            if not cfg.layer_is_sparse[l]:
                Ly.dense_gate, Ly.dense_up = self._q(b + "ffn_gate.weight"), self._q(b + "ffn_up.weight")
                Ly.dense_down = self._q(b + "ffn_down.weight")
                Ly.dense_gscale = gscale
            else:
                M = Ly.moe
                M.hidden, M.ff = cfg.hidden_size, cfg.moe_intermediate_size
                M.n_routed, M.n_shared, M.topk = cfg.n_routed_experts, cfg.n_shared_experts, cfg.num_experts_per_tok
                M.route_scale, M.global_scale = cfg.route_scale, gscale
                M.router_w, M.router_bias = self._f(b + "ffn_gate_inp.weight"), self._f(b + "exp_probs_b.bias")
                ex = self.experts[l]
                M.gate_type, M.gate_stride, M.gate = ex["gate"][0], ex["gate"][1], ex["gate"][2].data_ptr()
                M.up_type, M.up_stride, M.up = ex["up"][0], ex["up"][1], ex["up"][2].data_ptr()
                M.down_type, M.down_stride, M.down = ex["down"][0], ex["down"][1], ex["down"][2].data_ptr()
                for key, fld in (("ffn_gate_shexp", "sh_gate"), ("ffn_up_shexp", "sh_up"), ("ffn_down_shexp", "sh_down")):
                    t, shape, buf = self.t[b + key + ".weight"]
                    setattr(M, fld + "_type", t)
                    setattr(M, fld, buf.data_ptr())
                    setattr(M, fld + "_stride", buf.numel() // max(1, cfg.n_shared_experts))
                M.rank, M.world = self.rank, self.world
                M.expert_slot = None
        d = SepiaModelDesc()
        d.hidden, d.n_layers = cfg.hidden_size, n
        d.vocab, d.unpadded_vocab = cfg.vocab_size, cfg.unpadded_vocab_size
        d.d_rel, d.conv_k, d.window = cfg.d_rel, cfg.conv_kernel_size, cfg.sliding_window_size
        d.max_positions = self.max_positions
        d.eps, d.mup = cfg.rms_norm_eps, cfg.logits_mup_width_multiplier
        d.has_log_scaling = int(cfg.log_scaling_n_floor is not None)
        d.log_scaling_alpha = cfg.log_scaling_alpha
        d.log_scaling_n_floor = cfg.log_scaling_n_floor or 0
        d.embed, d.unembed = self._q("token_embd.weight"), self._q("output.weight")
        d.embed_norm, d.final_norm = self._f("token_embd_norm.weight"), self._f("output_norm.weight")
        d.layers = self._layers
        d.rank, d.world = self.rank, self.world
        self._desc = d
        h = C.c_void_p()
        ok(L.sepia_model_create(C.byref(d), C.byref(h)), "model_create")
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            try:
                load().sepia_model_destroy(self._h)
            except Exception:
                pass
            self._h = None

    def connect(self, group=None):
        """Expert sharding: all-gathers every rank's exchange-buffer IPC
        handle over torch.distributed (host objects only) and opens the
        peers' buffers. Call once on every rank before the first token."""
        if self.world == 1:
            return
        import torch.distributed as dist
        h = (C.c_char * 64)()
        ok(load().sepia_model_exchange_handle(self._h, h), "model_exchange_handle")
        allh = [None] * self.world
        dist.all_gather_object(allh, bytes(h), group=group)
        buf = (C.c_char * (64 * self.world)).from_buffer_copy(b"".join(allh))
        ok(load().sepia_model_connect(self._h, buf), "model_connect")

    # --------------------------------------------------------------- run
    def _st(self, stream=None) -> int:
        return (stream or torch.cuda.current_stream()).cuda_stream

    def reset(self, stream=None):
        ok(load().sepia_model_reset(self._h, self._st(stream)), "model_reset")

    def prefill(self, ids: torch.Tensor, want_logits: bool = True, stream=None):
        assert ids.dtype == torch.int32 and ids.is_cuda
        ok(load().sepia_model_prefill(self._h, ids.data_ptr(), ids.numel(), int(want_logits), self._st(stream)),
           "model_prefill")

    def decode(self, out_ids: torch.Tensor, n: int | None = None, stream=None):
        assert out_ids.dtype == torch.int32 and out_ids.is_cuda
        n = out_ids.numel() if n is None else n
        ok(load().sepia_model_decode(self._h, n, out_ids.data_ptr(), self._st(stream)), "model_decode")

    def logits(self, stream=None) -> torch.Tensor:
        """A copy of the last computed logits [unpadded_vocab]."""
        out = torch.empty(self.cfg.unpadded_vocab_size, dtype=torch.float32, device=self.device)
        ok(load().sepia_model_copy_logits(self._h, out.data_ptr(), self._st(stream)), "model_copy_logits")
        return out

    def position(self, stream=None) -> int:
        return int(load().sepia_model_position(self._h, self._st(stream)))

    def generate(self, prompt, n_gen: int, stream=None) -> np.ndarray:
        """Greedy ids: id 0 is the argmax of the prompt's last logits, id i
        the argmax after feeding id i-1 (real_generate's loop)."""
        ids = torch.as_tensor(np.asarray(prompt, np.int32), device=self.device)
        out = torch.empty(n_gen, dtype=torch.int32, device=self.device)
        self.reset(stream)
        self.prefill(ids, True, stream)
        self.decode(out, n_gen, stream)
        return out.cpu().numpy()
