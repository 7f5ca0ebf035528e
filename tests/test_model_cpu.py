"""CPU: the container reader/writer (sepia_b200/container.py) and the
greedy-decode golden fixtures (tests/golden/model_*.npz) against the
reference's own decoder when its checkout is present."""
import json
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_model_golden as G  # noqa: E402

from sepia_b200 import container as CT  # noqa: E402
from sepia_b200 import quants as Q  # noqa: E402


def test_config_resolution_rules():
    """config_load's precedence (src/sepia.c:476-533): layer_types over
    local_layer_ids over the every-6th default; mlp_layer_types over
    dense_mlp_idx; dense_intermediate_size over intermediate_size;
    moe_intermediate_size defaults to 3072; a null log_scaling_n_floor
    disables log scaling."""
    tc = CT.synth_text_config(n_layers=7)
    c = CT.ModelConfig.from_text_config(tc)
    assert c.layer_is_sliding == [(i + 1) % 3 != 0 for i in range(7)]
    t2 = dict(tc)
    del t2["layer_types"]
    t2["local_layer_ids"] = [0, 2]
    assert CT.ModelConfig.from_text_config(t2).layer_is_sliding == [True, False, True] + [False] * 4
    del t2["local_layer_ids"]
    assert CT.ModelConfig.from_text_config(t2).layer_is_sliding == [(i + 1) % 6 != 0 for i in range(7)]
    del t2["mlp_layer_types"]
    t2["dense_mlp_idx"] = 3
    assert CT.ModelConfig.from_text_config(t2).layer_is_sparse == [False] * 3 + [True] * 4
    del t2["dense_mlp_idx"]
    assert all(CT.ModelConfig.from_text_config(t2).layer_is_sparse)
    del t2["dense_intermediate_size"], t2["moe_intermediate_size"]
    t2["intermediate_size"] = 1024
    c2 = CT.ModelConfig.from_text_config(t2)
    assert c2.dense_intermediate_size == 1024 and c2.moe_intermediate_size == 3072
    t2["log_scaling_n_floor"] = None
    assert CT.ModelConfig.from_text_config(t2).log_scaling_n_floor is None
    with pytest.raises(ValueError):
        CT.ModelConfig.from_text_config({k: v for k, v in tc.items() if k != "hidden_size"})


def test_container_round_trip(tmp_path):
    tc = CT.synth_text_config(n_layers=3, n_experts=8, topk=2)
    types = CT.ModelTypes()
    d = CT.synth_container(tmp_path / "m", tc, types=types, seed=3)
    ct = CT.Container(d)
    cfg = ct.cfg
    specs = CT.resident_specs(cfg, types)
    assert set(ct.tensors) == {n for n, _, _ in specs}
    written = CT.synth_resident(cfg, types, 3)
    for name, t, shape in specs:
        tt, ss, buf = ct.resident(name)
        assert tt == t and list(ss) == list(shape)
        assert np.array_equal(buf, written[name][2]), name
        assert ct.tensors[name]["offset"] % 64 == 0
    idx = json.loads((Path(d) / "index.json").read_text())
    assert idx["n_experts_per_layer"] == 8 and set(idx["moe_layers"]) == {"1", "2"}
    for l in (1, 2):
        for slot, (rows, cols, t) in {"gate": (cfg.moe_intermediate_size, cfg.hidden_size, types.gate),
                                      "up": (cfg.moe_intermediate_size, cfg.hidden_size, types.up),
                                      "down": (cfg.hidden_size, cfg.moe_intermediate_size, types.down)}.items():
            tt, nb, ents = ct.expert_layer(l, slot)
            assert tt == t and nb == Q.row_bytes(t, cols) * rows
            raw = (Path(d) / CT.GGUF_DIR / ents[0]["part_file"]).read_bytes()
            assert raw[:4] == b"GGUF"
            for e in (0, 5, 7):
                assert ct.expert_bytes(l, slot, e) == raw[ents[e]["abs_offset"]:ents[e]["abs_offset"] + nb]
    ct.close()


@pytest.mark.parametrize("name", list(G.MODELS))
def test_golden_fixture_is_deterministic_and_reference_reproduces_it(tmp_path, oracle, name):
    fx = np.load(Path(G.HERE) / f"model_{name}.npz")
    d, prompt, digest = G.build(name, tmp_path / name)
    assert digest == str(fx["digest"]), "container bytes changed: regenerate the fixture"
    assert np.array_equal(prompt, fx["prompt"])
    if oracle.ref_lib() is None:
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    ids, logits = oracle.ref_generate(d, prompt, len(fx["ids"]))
    assert np.array_equal(ids, fx["ids"])
    assert np.array_equal(logits.view(np.uint32), fx["logits"].view(np.uint32))
