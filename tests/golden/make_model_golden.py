#!/usr/bin/env python3
"""Generates the greedy-decode golden fixtures tests/golden/model_<name>.npz
from the reference's own CPU decoder (real_load + real_forward_chunk +
real_generate's loop, rinaldofesta/sepia src/sepia.c:2647, 3345, 4114),
compiled in place by oracle/Makefile into oracle/_ref/libsepia_ref.so.

Each fixture holds the prompt, the container's checksum, the n_gen greedy
ids and the logits each id was taken from. The containers are small
synthetic models with the Inkling layer structure (dense + MoE layers,
sliding + global attention, tau != 1), written deterministically by
sepia_b200.container.synth_container, so a test can rebuild the exact same
bytes and compare its own decode with the reference's.

  MODELS["real_types"]      the real model's formats (IQ2_XS/IQ3_XXS
                            experts, K-quant attention), all in src/quants.c
  MODELS["baseline_types"]  BASELINE's Q2_K/Q3_K experts; the reference lacks
                            those two formats, so oracle/ref_shim.c supplies
                            their dequantization from the restatement pinned
                            to gguf-py 0.19.0 (everything else is the
                            reference's code)

Usage: python tests/golden/make_model_golden.py   (needs the reference checkout)
"""
from __future__ import annotations

import hashlib
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from sepia_b200 import container as CT  # noqa: E402
from sepia_b200 import quants as Q  # noqa: E402

MODELS = {
    "real_types": dict(
        text_config=CT.synth_text_config(),
        types=CT.ModelTypes(embed=Q.Q8_0, unembed=Q.Q6_K, attn=Q.Q4_K, dense=Q.Q5_K, gate=Q.IQ2_XS, up=Q.IQ2_XS,
                            down=Q.IQ3_XXS, shared=Q.Q5_K),
        seed=7, prompt_len=20, n_gen=32),
    "baseline_types": dict(
        text_config=CT.synth_text_config(n_layers=5, global_every=2, n_experts=32, topk=6),
        types=CT.ModelTypes(embed=Q.Q8_0, unembed=Q.Q6_K, attn=Q.Q4_K, dense=Q.Q4_K, gate=Q.Q2_K, up=Q.Q2_K,
                            down=Q.Q3_K, shared=Q.Q4_K),
        seed=11, prompt_len=16, n_gen=32),
}


def container_digest(d: Path) -> str:
    h = hashlib.sha256()
    for name in ("config.json", "resident.bin", "resident-manifest.json", "index.json"):
        h.update((d / name).read_bytes())
    for p in sorted((d / CT.GGUF_DIR).rglob("*.gguf")):
        h.update(p.read_bytes())
    return h.hexdigest()


def build(name: str, out_dir: Path) -> tuple[Path, np.ndarray, str]:
    spec = MODELS[name]
    d = CT.synth_container(out_dir, spec["text_config"], types=spec["types"], seed=spec["seed"])
    prompt = np.random.default_rng(spec["seed"]).integers(0, spec["text_config"]["vocab_size"],
                                                          spec["prompt_len"]).astype(np.int32)
    return Path(d), prompt, container_digest(Path(d))


def main():
    from oracle import oracle as O
    O.build()
    if O.ref_lib() is None:
        raise SystemExit("oracle/_ref not built: the reference checkout is needed")
    for name, spec in MODELS.items():
        with tempfile.TemporaryDirectory() as tmp:
            d, prompt, digest = build(name, Path(tmp) / name)
            ids, logits = O.ref_generate(d, prompt, spec["n_gen"])
            s = np.sort(logits, axis=1)
            print(f"{name}: ids {ids.tolist()} min top-2 margin {float((s[:, -1] - s[:, -2]).min()):.4f}")
            np.savez_compressed(HERE / f"model_{name}.npz", prompt=prompt, ids=ids, logits=logits,
                                digest=np.array(digest))


if __name__ == "__main__":
    main()
