"""CPU: the oracle's attention-layer composition (oracle/model_oracle.py
attn_chunk, built on or_banded_attn64 / or_rel_project / or_sconv_apply /
or_rmsnorm / or_linear) against the reference's own attn_forward_chunk
(src/sepia.c:1077-1276) compiled in place (oracle/_ref). Bit-exact: this is
what pins or_banded_attn, the restatement the GPU attention tests use as
their checker. Cases cover prefill then decode, sliding windows shorter
than the context, the relative band edge, GQA and log-scaling tau != 1."""
import numpy as np
import pytest


def _ref(oracle):
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    return R


CASES = {
    # hidden, H, Hkv, Dh, d_rel, E, K, sliding, window, has_log, n_floor, chunks
    "global_tau": (256, 4, 2, 64, 8, 16, 4, 0, 0, 1, 4, [5, 1, 1, 3]),
    "sliding_short_window": (128, 4, 4, 32, 4, 8, 4, 1, 6, 0, 1, [7, 1, 1, 1, 4]),
    "gqa_band_edge": (192, 6, 2, 32, 8, 5, 3, 0, 0, 1, 2, [3, 4, 1]),
    "dh_odd": (128, 4, 2, 40, 4, 12, 4, 1, 9, 0, 1, [10, 1, 2]),
}


@pytest.mark.parametrize("name", list(CASES))
def test_attn_chunk_matches_reference(oracle, name):
    from oracle import model_oracle as M
    R = _ref(oracle)
    hidden, H, Hkv, Dh, d_rel, E, K, sliding, window, has_log, n_floor, chunks = CASES[name]
    rng = np.random.default_rng(len(name))
    q_dim, kv_dim, r_dim = H * Dh, Hkv * Dh, H * d_rel
    f = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)
    lw = dict(is_sliding=bool(sliding), H=H, Hkv=Hkv, Dh=Dh, rel_extent=E,
              wq=f(q_dim, hidden, sc=0.1), wk=f(kv_dim, hidden, sc=0.1), wv=f(kv_dim, hidden, sc=0.1),
              wr=f(r_dim, hidden, sc=0.1), wo=f(hidden, q_dim, sc=0.05),
              q_norm=1 + f(Dh, sc=0.1), k_norm=1 + f(Dh, sc=0.1), rel_proj=f(d_rel, E, sc=0.3),
              k_sconv=f(kv_dim, K, sc=0.1), v_sconv=f(kv_dim, K, sc=0.1))
    cfg = dict(hidden=hidden, d_rel=d_rel, conv_k=K, eps=1e-6, window=window, has_log_scaling=bool(has_log),
               log_scaling_alpha=0.1, log_scaling_n_floor=n_floor)
    cap = sum(chunks)
    mine = dict(k=np.zeros((cap, kv_dim), np.float32), v=np.zeros((cap, kv_dim), np.float32),
                k_hist=np.zeros((K - 1) * kv_dim, np.float32), v_hist=np.zeros((K - 1) * kv_dim, np.float32))
    theirs = {k: v.copy() for k, v in mine.items()}
    pos = 0
    for T in chunks:
        x = f(T, hidden)
        got = M.attn_chunk(cfg, lw, mine, x, T, pos)
        want = np.empty((T, hidden), np.float32)
        R.ref_attn_chunk(hidden, H, Hkv, Dh, d_rel, E, K, int(sliding), window, np.float32(1e-6), int(has_log),
                         0.1, n_floor, lw["wq"], lw["wk"], lw["wv"], lw["wr"], lw["wo"], lw["q_norm"], lw["k_norm"],
                         lw["rel_proj"], lw["k_sconv"], lw["v_sconv"], theirs["k"], theirs["v"], theirs["k_hist"],
                         theirs["v_hist"], x, T, pos, want)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (name, pos)
        for key in mine:
            assert np.array_equal(mine[key], theirs[key]), key
        pos += T
