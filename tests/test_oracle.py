"""CPU: pin the oracle (oracle/*.c) before trusting it.

1. bitwise against this repo's committed gguf-py golden fixtures (all 13 types);
2. bitwise against the reference's own fixtures (tools/fixtures/quants);
3. bitwise against the reference's src/quants.c and src/sepia.c compiled in
   place (oracle/_ref), on fresh random blocks and inputs.
"""
import numpy as np
import pytest

from golden_io import golden_files, read_fixture, sqlx_parts


@pytest.mark.parametrize("path", golden_files("sqfx"), ids=lambda p: p.stem)
def test_dequant_matches_gguf_golden(oracle, path):
    fx = read_fixture(path)
    n = fx["n_blocks"] * fx["block_elems"]
    assert oracle.block_size(fx["type"]) == fx["block_elems"]
    assert oracle.type_size(fx["type"]) == fx["block_bytes"]
    got = oracle.dequantize(fx["type"], fx["raw"], n)
    assert np.array_equal(got.view(np.uint32), fx["expect"].view(np.uint32))


@pytest.mark.parametrize("path", golden_files("sqlx"), ids=lambda p: p.stem)
def test_qlinear_matches_golden(oracle, path):
    fx = read_fixture(path)
    w, x, y = sqlx_parts(fx, oracle.row_bytes(fx["type"], fx["in"]))
    got = oracle.qlinear(fx["type"], w, fx["out"], fx["in"], x)
    assert np.array_equal(got.view(np.uint32), y.view(np.uint32))


def test_reference_fixtures(oracle, reference_dir):
    files = sorted((reference_dir / "tools" / "fixtures" / "quants").glob("*.bin"))
    assert len(files) == 9
    for p in files:
        fx = read_fixture(p)
        if fx["kind"] == "sqfx":
            n = fx["n_blocks"] * fx["block_elems"]
            got = oracle.dequantize(fx["type"], fx["raw"], n)
            assert np.array_equal(got.view(np.uint32), fx["expect"].view(np.uint32)), p.name
        else:
            w, x, y = sqlx_parts(fx, oracle.row_bytes(fx["type"], fx["in"]))
            got = oracle.qlinear(fx["type"], w, fx["out"], fx["in"], x)
            assert np.array_equal(got.view(np.uint32), y.view(np.uint32)), p.name


def _ref(oracle):
    R = oracle.ref_lib()
    if R is None:
        pytest.skip("oracle/_ref not built (reference checkout absent)")
    return R


@pytest.mark.parametrize("t", [0, 1, 8, 12, 13, 14, 17, 18, 23])
def test_dequant_matches_reference_quants_c(oracle, t):
    R = _ref(oracle)
    from sepia_b200 import synth
    rng = np.random.default_rng(100 + t)
    e = oracle.block_size(t)
    nb = 4096 if e == 1 else (64 if e == 32 else 24)
    raw = synth.blocks_host(rng, t, nb)
    if t not in (0, 1):   # widen the scale fields to every finite half, as the reference fixtures do
        from sepia_b200 import quants as Q
        bb = Q.block_bytes(t)
        r2 = raw.reshape(nb, bb)
        for off in Q.F16_FIELDS[t]:
            bits = rng.integers(0, 0x7C00, size=nb, dtype=np.uint16) | (rng.integers(0, 2, nb, dtype=np.uint16) << 15)
            r2[:, off:off + 2] = bits.view(np.uint8).reshape(nb, 2)
    n = nb * e
    want = np.empty(n, np.float32)
    assert R.ref_dequantize_row(t, raw.ctypes.data, want, n) == 1
    got = oracle.dequantize(t, raw, n)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t", [8, 12, 13, 14, 17, 18, 23])
def test_qlinear_matches_reference(oracle, t):
    R = _ref(oracle)
    from sepia_b200 import synth
    rng = np.random.default_rng(7 + t)
    out_dim, in_dim = 16, 1024
    w = synth.matrix_host(rng, t, out_dim, in_dim)
    x = rng.standard_normal(in_dim).astype(np.float32)
    want = np.empty(out_dim, np.float32)
    assert R.ref_qlinear(t, w.ctypes.data, out_dim, in_dim, x, want, 2) == 1
    got = oracle.qlinear(t, w, out_dim, in_dim, x, nthreads=3)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("seed", range(8))
def test_route_select_matches_reference(oracle, seed):
    R = _ref(oracle)
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal(258) * 2).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, 256).astype(np.float32)
    if seed % 2:   # force exact ties in the selection score
        logits[10] = logits[200]
        bias[10] = bias[200]
    i1, w1 = oracle.route_select(logits, bias, 256, 2, 6, 8.0, 1.0)
    i2 = np.empty(6, np.int32)
    w2 = np.empty(8, np.float32)
    R.ref_route_select(256, 2, 6, 8.0, 1.0, logits, bias, i2, w2)
    assert np.array_equal(i1, i2)
    assert np.array_equal(w1.view(np.uint32), w2.view(np.uint32))


def test_topk_tie_rule(oracle):
    s = np.zeros(16, np.float32)
    s[[3, 7, 9]] = 1.0
    assert list(oracle.topk_scores(s, 4)) == [3, 7, 9, 0]


def test_rmsnorm_and_sconv_match_reference(oracle):
    R = _ref(oracle)
    rng = np.random.default_rng(3)
    x = rng.standard_normal(1024).astype(np.float32)
    w = rng.standard_normal(1024).astype(np.float32)
    a = np.empty_like(x)
    b = np.empty_like(x)
    R.ref_rmsnorm(x, w, 1024, np.float32(1e-5), a)
    oracle.lib().or_rmsnorm(x, w, 1024, np.float32(1e-5), b)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    C_, K, T = 64, 4, 5
    wc = (rng.standard_normal(C_ * K) * 0.1).astype(np.float32)
    h1 = rng.standard_normal((K - 1) * C_).astype(np.float32)
    h2 = h1.copy()
    inp = rng.standard_normal(T * C_).astype(np.float32)
    o1 = np.empty_like(inp)
    o2 = np.empty_like(inp)
    R.ref_sconv_apply(wc, C_, K, h1, inp, T, o1)
    oracle.lib().or_sconv_apply(wc, C_, K, h2, inp, T, o2)
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))
    assert np.array_equal(h1.view(np.uint32), h2.view(np.uint32))
