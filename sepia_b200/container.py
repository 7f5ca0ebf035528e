"""The reference's model container: config.json, resident.bin +
resident-manifest.json, the sepia-index JSON and the GGUF parts that hold
the routed experts (format: docs/container.md:123-257 of rinaldofesta/sepia;
reader: real_load, src/sepia.c:2647-2860).

  ModelConfig.load(path)      text_config fields, resolved like config_load
                              (src/sepia.c:455-553)
  Container(dir)              read access: resident tensors by name (zero
                              copy, mmap) and expert slabs by (layer, slot, e)
  write_container(...)        writes the four pieces from numpy arrays
  synth_container(...)        a seeded random model in BASELINE's weight
                              distributions, written as a container

Directory layout (what real_load opens, src/sepia.c:2657-2705):
  <dir>/config.json
  <dir>/resident.bin, <dir>/resident-manifest.json
  <dir>/index.json, <dir>/inkling-gguf/<part_file>
Shapes follow GGUF: dims[0] is the fastest axis, so a [rows, cols] matrix is
recorded as [cols, rows] (src/sepia.c:1930-1949).
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import quants as Q
from . import synth

GGUF_DIR = "inkling-gguf"


# --------------------------------------------------------------- config
@dataclass
class ModelConfig:
    hidden_size: int
    num_hidden_layers: int
    vocab_size: int
    unpadded_vocab_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    swa_num_attention_heads: int
    swa_num_key_value_heads: int
    swa_head_dim: int
    sliding_window_size: int
    layer_is_sliding: list
    layer_is_sparse: list
    d_rel: int
    rel_extent: int
    conv_kernel_size: int
    dense_intermediate_size: int
    moe_intermediate_size: int
    n_routed_experts: int
    num_experts_per_tok: int
    n_shared_experts: int
    route_scale: float
    logits_mup_width_multiplier: float
    rms_norm_eps: float
    log_scaling_alpha: float
    log_scaling_n_floor: int | None
    raw: dict = field(default_factory=dict, repr=False)

    # per-layer attention geometry (real_fill_layer, src/sepia.c:2929-2937)
    def heads(self, l):
        if self.layer_is_sliding[l]:
            return self.swa_num_attention_heads, self.swa_num_key_value_heads, self.swa_head_dim
        return self.num_attention_heads, self.num_key_value_heads, self.head_dim

    def layer_rel_extent(self, l):
        return self.sliding_window_size if self.layer_is_sliding[l] else self.rel_extent

    @classmethod
    def from_text_config(cls, tc: dict) -> "ModelConfig":
        def req(k):
            if tc.get(k) is None:
                raise ValueError(f"config.json: missing required text_config field '{k}'")
            return tc[k]
        n = int(req("num_hidden_layers"))
        lt = tc.get("layer_types")
        if isinstance(lt, list):
            if len(lt) != n:
                raise ValueError("config.json: layer_types length differs from num_hidden_layers")
            sliding = [t == "hybrid_sliding" for t in lt]
        elif isinstance(tc.get("local_layer_ids"), list):
            sliding = [False] * n
            for i in tc["local_layer_ids"]:
                sliding[int(i)] = True
        else:
            sliding = [((i + 1) % 6) != 0 for i in range(n)]
        mlt = tc.get("mlp_layer_types")
        if isinstance(mlt, list):
            if len(mlt) != n:
                raise ValueError("config.json: mlp_layer_types length differs from num_hidden_layers")
            sparse = [t == "sparse" for t in mlt]
        else:
            dmi = tc.get("dense_mlp_idx")
            dmi = 0 if dmi is None else int(dmi)
            sparse = [i >= dmi for i in range(n)]
        dense_ff = tc.get("dense_intermediate_size")
        dense_ff = int(dense_ff) if dense_ff is not None else int(req("intermediate_size"))
        moe_ff = tc.get("moe_intermediate_size")
        moe_ff = 3072 if moe_ff is None else int(moe_ff)
        floor = tc.get("log_scaling_n_floor")
        return cls(
            hidden_size=int(req("hidden_size")), num_hidden_layers=n, vocab_size=int(req("vocab_size")),
            unpadded_vocab_size=int(req("unpadded_vocab_size")),
            num_attention_heads=int(req("num_attention_heads")), num_key_value_heads=int(req("num_key_value_heads")),
            head_dim=int(req("head_dim")), swa_num_attention_heads=int(req("swa_num_attention_heads")),
            swa_num_key_value_heads=int(req("swa_num_key_value_heads")), swa_head_dim=int(req("swa_head_dim")),
            sliding_window_size=int(req("sliding_window_size")), layer_is_sliding=sliding, layer_is_sparse=sparse,
            d_rel=int(req("d_rel")), rel_extent=int(req("rel_extent")), conv_kernel_size=int(req("conv_kernel_size")),
            dense_intermediate_size=dense_ff, moe_intermediate_size=moe_ff,
            n_routed_experts=int(req("n_routed_experts")), num_experts_per_tok=int(req("num_experts_per_tok")),
            n_shared_experts=int(req("n_shared_experts")), route_scale=float(req("route_scale")),
            logits_mup_width_multiplier=float(req("logits_mup_width_multiplier")),
            rms_norm_eps=float(req("rms_norm_eps")), log_scaling_alpha=float(req("log_scaling_alpha")),
            log_scaling_n_floor=None if floor is None else int(floor), raw=dict(tc))

    @classmethod
    def load(cls, path) -> "ModelConfig":
        root = json.loads(Path(path).read_text())
        if "text_config" not in root:
            raise ValueError("config.json: missing text_config")
        return cls.from_text_config(root["text_config"])


# ------------------------------------------------------------------ types
@dataclass
class ModelTypes:
    """Quant formats of a synthetic model (Q2_K/Q3_K
    experts, Q4_K elsewhere)."""
    embed: int = Q.Q4_K
    unembed: int = Q.Q4_K
    attn: int = Q.Q4_K
    dense: int = Q.Q4_K
    gate: int = Q.Q2_K
    up: int = Q.Q2_K
    down: int = Q.Q3_K
    shared: int = Q.Q4_K


def resident_specs(cfg: ModelConfig, types: ModelTypes):
    """(name, ggml_type, gguf_shape) of every resident tensor real_load
    resolves (src/sepia.c:2757-2800), in file order."""
    H = cfg.hidden_size
    K = cfg.conv_kernel_size
    out = [("token_embd.weight", types.embed, [H, cfg.vocab_size]),
           ("token_embd_norm.weight", Q.F32, [H]),
           ("output_norm.weight", Q.F32, [H]),
           ("output.weight", types.unembed, [H, cfg.vocab_size])]
    ns = cfg.n_shared_experts
    for l in range(cfg.num_hidden_layers):
        nh, nkv, dh = cfg.heads(l)
        E = cfg.layer_rel_extent(l)
        b = f"blk.{l}."
        out += [(b + "attn_norm.weight", Q.F32, [H]), (b + "ffn_norm.weight", Q.F32, [H]),
                (b + "attn_q_norm.weight", Q.F32, [dh]), (b + "attn_k_norm.weight", Q.F32, [dh]),
                (b + "attn_rel_proj.weight", Q.F32, [E, cfg.d_rel]),
                (b + "shortconv_k.weight", Q.F32, [K, nkv * dh]), (b + "shortconv_v.weight", Q.F32, [K, nkv * dh]),
                (b + "shortconv_attn.weight", Q.F32, [K, H]), (b + "shortconv_mlp.weight", Q.F32, [K, H]),
                (b + "attn_q.weight", types.attn, [H, nh * dh]), (b + "attn_k.weight", types.attn, [H, nkv * dh]),
                (b + "attn_v.weight", types.attn, [H, nkv * dh]),
                (b + "attn_r.weight", types.attn, [H, nh * cfg.d_rel]),
                (b + "attn_output.weight", types.attn, [nh * dh, H])]
        if cfg.layer_is_sparse[l]:
            ff = cfg.moe_intermediate_size
            out += [(b + "ffn_gate_inp.weight", Q.F32, [H, cfg.n_routed_experts + ns]),
                    (b + "exp_probs_b.bias", Q.F32, [cfg.n_routed_experts]),
                    (b + "ffn_gscale.weight", Q.F32, [1]),
                    (b + "ffn_gate_shexp.weight", types.shared, [H, ff, ns]),
                    (b + "ffn_up_shexp.weight", types.shared, [H, ff, ns]),
                    (b + "ffn_down_shexp.weight", types.shared, [ff, H, ns])]
        else:
            ff = cfg.dense_intermediate_size
            out += [(b + "ffn_gate.weight", types.dense, [H, ff]), (b + "ffn_up.weight", types.dense, [H, ff]),
                    (b + "ffn_down.weight", types.dense, [ff, H]), (b + "ffn_gscale.weight", Q.F32, [1])]
    return out


def tensor_nbytes(t: int, shape) -> int:
    n_rows = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    return Q.row_bytes(t, shape[0]) * n_rows


# ------------------------------------------------------------------ GGUF
def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: Path, tensors, alignment: int = 32):
    """A GGUF v3 file (header + tensor infos + aligned data). tensors:
    [(name, ggml_type, gguf_shape, bytes)]. Returns {name: absolute data offset}."""
    offs, run = [], 0
    for _, _, _, data in tensors:
        run = (run + alignment - 1) // alignment * alignment
        offs.append(run)
        run += len(data)
    hdr = bytearray(b"GGUF" + struct.pack("<I", 3) + struct.pack("<Q", len(tensors)) + struct.pack("<Q", 2))
    hdr += _gguf_str("general.architecture") + struct.pack("<I", 8) + _gguf_str("sepia-synthetic")
    hdr += _gguf_str("general.alignment") + struct.pack("<I", 4) + struct.pack("<I", alignment)
    for (name, t, shape, _), off in zip(tensors, offs):
        hdr += _gguf_str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        hdr += struct.pack("<I", t) + struct.pack("<Q", off)
    data_start = (len(hdr) + alignment - 1) // alignment * alignment
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        f.write(hdr)
        f.write(b"\0" * (data_start - len(hdr)))
        pos = data_start
        for (_, _, _, data), off in zip(tensors, offs):
            f.write(b"\0" * (data_start + off - pos))
            f.write(data)
            pos = data_start + off + len(data)
    return {name: data_start + off for (name, _, _, _), off in zip(tensors, offs)}


# ------------------------------------------------------------ container
def write_container(out_dir, text_config: dict, resident: dict, experts: dict, types_of_experts: dict,
                    part_file: str = "SYNTH/synth-00001-of-00001.gguf"):
    """resident: name -> (ggml_type, gguf_shape, uint8 array);
    experts: layer -> {"gate"|"up"|"down": uint8 array of n_experts slabs};
    types_of_experts: slot -> ggml_type."""
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    (out / "config.json").write_text(json.dumps({"text_config": text_config}, indent=1))
    entries, pos = [], 0
    with open(out / "resident.bin", "wb") as f:
        for name, (t, shape, data) in resident.items():
            pad = (-pos) % 64
            f.write(b"\0" * pad)
            pos += pad
            f.write(np.ascontiguousarray(data).view(np.uint8).tobytes())
            entries.append({"name": name, "ggml_type": int(t), "offset": pos, "nbytes": int(data.nbytes),
                            "shape": [int(d) for d in shape]})
            pos += int(data.nbytes)
    (out / "resident-manifest.json").write_text(json.dumps({"tensors": entries}, indent=1))
    cfg = ModelConfig.from_text_config(text_config)
    H, ff, n_e = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts
    gguf, shapes = [], {"gate": [H, ff, n_e], "up": [H, ff, n_e], "down": [ff, H, n_e]}
    for l in sorted(experts):
        for slot in ("gate", "up", "down"):
            gguf.append((f"blk.{l}.ffn_{slot}_exps.weight", types_of_experts[slot], shapes[slot],
                         np.ascontiguousarray(experts[l][slot]).tobytes()))
    offs = write_gguf(out / GGUF_DIR / part_file, gguf)
    moe_layers = {}
    for l in sorted(experts):
        d = {}
        for slot in ("gate", "up", "down"):
            t = types_of_experts[slot]
            nb = tensor_nbytes(t, shapes[slot][:2])
            base = offs[f"blk.{l}.ffn_{slot}_exps.weight"]
            d[slot] = {"bytes_per_expert": nb, "experts": [
                {"part_file": part_file, "abs_offset": base + e * nb, "nbytes": nb, "ggml_type": int(t)}
                for e in range(n_e)]}
        moe_layers[str(l)] = d
    (out / "index.json").write_text(json.dumps({"n_experts_per_layer": n_e, "parts": [{"part_file": part_file}],
                                                "moe_layers": moe_layers}))
    return out


class Container:
    """Read access to a container directory (real_load's inputs)."""

    def __init__(self, path, index_name: str = "index.json"):
        self.dir = Path(path)
        self.cfg = ModelConfig.load(self.dir / "config.json")
        self._res_f = open(self.dir / "resident.bin", "rb")
        size = os.fstat(self._res_f.fileno()).st_size
        self._res = mmap.mmap(self._res_f.fileno(), size, access=mmap.ACCESS_READ) if size else b""
        man = json.loads((self.dir / "resident-manifest.json").read_text())
        self.tensors = {}
        for t in man["tensors"]:
            if t["offset"] < 0 or t["offset"] + t["nbytes"] > size:
                raise ValueError(f"resident tensor {t['name']} exceeds resident.bin")
            self.tensors[t["name"]] = t
        self.index = json.loads((self.dir / index_name).read_text())
        if self.index["n_experts_per_layer"] != self.cfg.n_routed_experts:
            raise ValueError("index: n_experts_per_layer disagrees with n_routed_experts")
        self._parts = {}

    def close(self):
        for f in self._parts.values():
            f.close()
        self._parts = {}

    def resident(self, name: str):
        """(ggml_type, gguf_shape, uint8 array view into resident.bin)."""
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"resident-manifest: missing tensor '{name}'")
        want = tensor_nbytes(t["ggml_type"], t["shape"]) if t["ggml_type"] not in (Q.F32,) else \
            4 * int(np.prod(t["shape"]))
        if want != t["nbytes"]:
            raise ValueError(f"resident tensor '{name}': nbytes disagrees with shape/type")
        buf = np.frombuffer(self._res, dtype=np.uint8, count=t["nbytes"], offset=t["offset"])
        return t["ggml_type"], t["shape"], buf

    def f32(self, name: str) -> np.ndarray:
        t, shape, buf = self.resident(name)
        if t != Q.F32:
            raise ValueError(f"resident tensor '{name}': expected F32, got {t}")
        return buf.view(np.float32)

    def expert_layer(self, layer: int, slot: str):
        """(ggml_type, nbytes per expert, [entry...]) of one layer's slot."""
        ents = self.index["moe_layers"][str(layer)][slot]["experts"]
        t = ents[0]["ggml_type"]
        nb = ents[0]["nbytes"]
        for e in ents:
            if e["ggml_type"] != t or e["nbytes"] != nb:
                raise ValueError(f"index: layer {layer} {slot}: experts differ in type or size")
        return t, nb, ents

    def expert_bytes(self, layer: int, slot: str, e: int) -> bytes:
        ent = self.index["moe_layers"][str(layer)][slot]["experts"][e]
        pf = ent["part_file"]
        if pf not in self._parts:
            self._parts[pf] = open(self.dir / GGUF_DIR / pf, "rb")
        f = self._parts[pf]
        data = os.pread(f.fileno(), ent["nbytes"], ent["abs_offset"])
        if len(data) != ent["nbytes"]:
            raise ValueError(f"short read of layer {layer} {slot} expert {e}")
        return data


# -------------------------------------------------------------- synthetic
def synth_text_config(hidden=512, n_layers=4, vocab=512, unpadded=500, heads=4, kv_heads=2, head_dim=64,
                      swa_heads=4, swa_kv_heads=2, swa_head_dim=64, window=16, d_rel=8, rel_extent=24, conv_k=4,
                      dense_ff=512, moe_ff=256, n_experts=16, topk=4, n_shared=2, route_scale=8.0, mup=4.0,
                      eps=1e-6, log_alpha=0.1, log_floor=8, n_dense=1, global_every=3):
    """text_config of a small model with the Inkling layer structure: the
    first n_dense layers dense, every global_every-th layer global."""
    return {
        "hidden_size": hidden, "num_hidden_layers": n_layers, "vocab_size": vocab, "unpadded_vocab_size": unpadded,
        "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
        "swa_num_attention_heads": swa_heads, "swa_num_key_value_heads": swa_kv_heads, "swa_head_dim": swa_head_dim,
        "sliding_window_size": window,
        "layer_types": ["hybrid" if (i + 1) % global_every == 0 else "hybrid_sliding" for i in range(n_layers)],
        "mlp_layer_types": ["dense" if i < n_dense else "sparse" for i in range(n_layers)],
        "d_rel": d_rel, "rel_extent": rel_extent, "conv_kernel_size": conv_k, "dense_intermediate_size": dense_ff,
        "moe_intermediate_size": moe_ff, "n_routed_experts": n_experts, "num_experts_per_tok": topk,
        "n_shared_experts": n_shared, "route_scale": route_scale, "logits_mup_width_multiplier": mup,
        "rms_norm_eps": eps, "log_scaling_alpha": log_alpha, "log_scaling_n_floor": log_floor}


def config5_text_config(n_layers: int = 66) -> dict:
    """the Inkling shape with hidden 7168, 256
    experts (top 6, 2 shared, ff 2048), 64 query / 8 KV heads of 128 in
    every layer, sliding window 4096 (every 6th layer global, rel_extent
    256), the first 2 layers dense, vocabulary 200k. n_layers truncates the
    66-layer stack (24 on one GPU). Fields the configuration leaves open take
    the real model's values (d_rel 16, kernel 4, mup 24, eps 1e-6, log
    scaling alpha 0.1 / floor 128000); the dense width is 4 x 4608."""
    return {
        "hidden_size": 7168, "num_hidden_layers": n_layers, "vocab_size": 200064, "unpadded_vocab_size": 200000,
        "num_attention_heads": 64, "num_key_value_heads": 8, "head_dim": 128,
        "swa_num_attention_heads": 64, "swa_num_key_value_heads": 8, "swa_head_dim": 128,
        "sliding_window_size": 4096,
        "layer_types": ["hybrid" if (i + 1) % 6 == 0 else "hybrid_sliding" for i in range(n_layers)],
        "mlp_layer_types": ["dense" if i < 2 else "sparse" for i in range(n_layers)],
        "d_rel": 16, "rel_extent": 256, "conv_kernel_size": 4, "dense_intermediate_size": 18432,
        "moe_intermediate_size": 2048, "n_routed_experts": 256, "num_experts_per_tok": 6, "n_shared_experts": 2,
        "route_scale": 8.0, "logits_mup_width_multiplier": 24.0, "rms_norm_eps": 1e-6,
        "log_scaling_alpha": 0.1, "log_scaling_n_floor": 128000}


def token_bytes(cfg: ModelConfig, types: ModelTypes, ctx: int) -> dict:
    """Algorithmic HBM bytes of one decode token at context ctx, per part:
    every weight the token reads once (attention projections, router, the
    top-k routed and all shared experts, dense MLPs, one embedding row, the
    unpadded logits head) plus the fp32 K/V cache rows attention reads."""
    H = cfg.hidden_size
    rb = Q.row_bytes
    attn = kv = moe = dense = 0
    for l in range(cfg.num_hidden_layers):
        nh, nkv, dh = cfg.heads(l)
        attn += (rb(types.attn, H) * (nh * dh + 2 * nkv * dh + nh * cfg.d_rel) + rb(types.attn, nh * dh) * H
                 + 4 * cfg.d_rel * cfg.layer_rel_extent(l))
        span = min(ctx, cfg.sliding_window_size) if cfg.layer_is_sliding[l] else ctx
        kv += 2 * 4 * nkv * dh * span
        if cfg.layer_is_sparse[l]:
            ff = cfg.moe_intermediate_size
            e = rb(types.gate, H) * ff + rb(types.up, H) * ff + rb(types.down, ff) * H
            sh = 2 * rb(types.shared, H) * ff + rb(types.shared, ff) * H
            moe += 4 * (cfg.n_routed_experts + cfg.n_shared_experts) * H + cfg.num_experts_per_tok * e \
                + cfg.n_shared_experts * sh
        else:
            ff = cfg.dense_intermediate_size
            dense += 2 * rb(types.dense, H) * ff + rb(types.dense, ff) * H
    head = rb(types.unembed, H) * cfg.unpadded_vocab_size + rb(types.embed, H)
    return {"attention": attn, "kv_cache": kv, "moe": moe, "dense": dense, "head": head,
            "total": attn + kv + moe + dense + head}


def synth_resident(cfg: ModelConfig, types: ModelTypes, seed: int):
    """name -> (type, shape, uint8 array), seeded. Quantized blocks follow
    BASELINE's distributions (uniform bytes, fp16 scales in [1e-3, 4e-3]);
    f32 tensors: norms 1 + N(0, 0.1), router N(0, 0.02), bias U(-0.1, 0.1),
    relative-position band N(0, 0.02), convolutions N(0, 0.1), global
    scales 1."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, t, shape in resident_specs(cfg, types):
        if t == Q.F32:
            n = int(np.prod(shape))
            if name.endswith("norm.weight"):
                a = 1.0 + rng.standard_normal(n) * 0.1
            elif name.endswith("ffn_gate_inp.weight"):
                a = rng.standard_normal(n) * 0.02
            elif name.endswith("exp_probs_b.bias"):
                a = rng.uniform(-0.1, 0.1, n)
            elif name.endswith("ffn_gscale.weight"):
                a = np.ones(n)
            elif name.endswith("attn_rel_proj.weight"):
                a = rng.standard_normal(n) * 0.02
            else:
                a = rng.standard_normal(n) * 0.1
            out[name] = (t, shape, a.astype(np.float32).view(np.uint8))
        else:
            n_blocks = tensor_nbytes(t, shape) // Q.block_bytes(t)
            out[name] = (t, shape, synth.blocks_host(rng, t, n_blocks))
    return out


def synth_container(out_dir, text_config: dict, types: ModelTypes | None = None, seed: int = 7):
    """Writes a seeded random container of the given configuration."""
    types = types or ModelTypes()
    cfg = ModelConfig.from_text_config(text_config)
    resident = synth_resident(cfg, types, seed)
    rng = np.random.default_rng(seed + 1)
    H, ff, n_e = cfg.hidden_size, cfg.moe_intermediate_size, cfg.n_routed_experts
    experts = {}
    for l in range(cfg.num_hidden_layers):
        if not cfg.layer_is_sparse[l]:
            continue
        experts[l] = {
            "gate": synth.blocks_host(rng, types.gate, n_e * Q.row_bytes(types.gate, H) * ff // Q.block_bytes(types.gate)),
            "up": synth.blocks_host(rng, types.up, n_e * Q.row_bytes(types.up, H) * ff // Q.block_bytes(types.up)),
            "down": synth.blocks_host(rng, types.down, n_e * Q.row_bytes(types.down, ff) * H // Q.block_bytes(types.down))}
    return write_container(out_dir, text_config, resident, experts,
                           {"gate": types.gate, "up": types.up, "down": types.down})
