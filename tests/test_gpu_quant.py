"""GPU: dequant bit-exactness and quantized matvec parity against the oracle.

Tolerance: max relative error <= 1e-4 with the reference's floored
denominator (src/sepia.c:4584-4589), tighter than the reference's 2e-4 gate.
"""
import numpy as np
import pytest

from golden_io import golden_files, read_fixture, sqlx_parts
from sepia_b200 import quants as Q
from sepia_b200 import synth

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def torch_cuda(lib):
    import torch
    return torch


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("path", golden_files("sqfx"), ids=lambda p: p.stem)
def test_dequant_bitwise_golden(torch_cuda, path):
    from sepia_b200 import ops
    torch = torch_cuda
    fx = read_fixture(path)
    n = fx["n_blocks"] * fx["block_elems"]
    got = ops.dequant(fx["type"], _dev(torch, fx["raw"]), n).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), fx["expect"].view(np.uint32))


@pytest.mark.parametrize("t", Q.QUANT_TYPES, ids=lambda t: Q.NAMES[t])
def test_dequant_bitwise_unaligned(torch_cuda, oracle, t):
    """Blocks starting at every byte offset 0..15 of a buffer."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(t)
    nb = 24 if Q.block_elems(t) == 256 else 64
    raw = synth.blocks_host(rng, t, nb)
    n = nb * Q.block_elems(t)
    want = oracle.dequantize(t, raw, n)
    buf = torch.zeros(raw.size + 64, dtype=torch.uint8, device="cuda")
    for off in (0, 1, 2, 3, 6, 10, 15):
        buf[off:off + raw.size] = _dev(torch, raw)
        got = torch.empty(n, dtype=torch.float32, device="cuda")
        from sepia_b200.lib import load, ok
        ok(load().sepia_cuda_dequant(t, buf.data_ptr() + off, got.data_ptr(), n, None))
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32)), off


@pytest.mark.parametrize("path", golden_files("sqlx"), ids=lambda p: p.stem)
def test_matvec_golden_sqlx(torch_cuda, oracle, path):
    from sepia_b200 import ops
    torch = torch_cuda
    fx = read_fixture(path)
    w, x, y = sqlx_parts(fx, oracle.row_bytes(fx["type"], fx["in"]))
    got = ops.matvec_q(fx["type"], _dev(torch, w), _dev(torch, x), fx["out"], fx["in"]).cpu().numpy()
    assert oracle.rel_err(got, y) <= TOL


SHAPES = [(1, 256), (3, 512), (17, 768), (64, 2048), (130, 7168), (33, 9216), (40, 18432), (24, 20480)]


@pytest.mark.parametrize("t", Q.ALL_TYPES, ids=lambda t: Q.NAMES[t])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}")
def test_matvec_vs_oracle(torch_cuda, oracle, t, shape):
    from sepia_b200 import ops
    torch = torch_cuda
    out_dim, in_dim = shape
    rng = np.random.default_rng(out_dim * 31 + in_dim + t)
    w = synth.matrix_host(rng, t, out_dim, in_dim)
    x = rng.standard_normal(in_dim).astype(np.float32)
    want = oracle.qlinear(t, w, out_dim, in_dim, x, nthreads=4)
    got = ops.matvec_q(t, _dev(torch, w), _dev(torch, x), out_dim, in_dim).cpu().numpy()
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("t", [Q.Q2_K, Q.Q3_K, Q.Q4_K, Q.IQ2_XS, Q.Q8_0, Q.F16])
@pytest.mark.parametrize("off", [2, 6, 8, 14])
def test_matvec_unaligned_base(torch_cuda, oracle, t, off):
    """Weights at a byte offset into a buffer (the ABI's w_off)."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(off + 100 * t)
    out_dim, in_dim = 40, 1536 if Q.block_elems(t) > 1 else 1000
    w = synth.matrix_host(rng, t, out_dim, in_dim)
    x = rng.standard_normal(in_dim).astype(np.float32)
    want = oracle.qlinear(t, w, out_dim, in_dim, x)
    buf = torch.zeros(w.size + 64, dtype=torch.uint8, device="cuda")
    buf[off:off + w.size] = _dev(torch, w)
    got = ops.matvec_q(t, buf, _dev(torch, x), out_dim, in_dim, w_offset=off).cpu().numpy()
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("t", [Q.IQ1_S, Q.IQ2_XXS, Q.IQ2_XS, Q.IQ3_XXS, Q.Q2_K])
@pytest.mark.parametrize("n_vec", [2, 4, 5, 16])
def test_matvec_batched(torch_cuda, oracle, t, n_vec):
    """BASELINE configuration 3 batches (smaller, ragged row count; n_vec 5
    leaves a partial vector group). Batch 1 of these formats runs on the
    tensor-core engine (exact integer dots), the batches on the CUDA-core
    kernel (fp32 part sums): both stay within the tolerance of the oracle
    and of each other."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(n_vec + t)
    out_dim, in_dim = 100, 7168
    w = synth.matrix_host(rng, t, out_dim, in_dim)
    X = rng.standard_normal((n_vec, in_dim)).astype(np.float32)
    wd = _dev(torch, w)
    got = ops.matvec_q(t, wd, _dev(torch, X), out_dim, in_dim).cpu().numpy()
    for v in range(n_vec):
        want = oracle.qlinear(t, w, out_dim, in_dim, X[v])
        assert oracle.rel_err(got[v], want) <= TOL
        if t != Q.Q2_K:
            one = ops.matvec_q(t, wd, _dev(torch, np.ascontiguousarray(X[v])), out_dim, in_dim).cpu().numpy()
            assert oracle.rel_err(one, got[v]) <= TOL


@pytest.mark.parametrize("t", [Q.IQ1_S, Q.IQ2_XXS, Q.IQ3_XXS])
@pytest.mark.parametrize("n_vec", [3, 5])
def test_matvec_vector_pairs(torch_cuda, oracle, t, n_vec):
    """Batches of these formats with >= 4096 rows run on the tensor-core
    engine two vectors per pass (MMA columns 0-3 and 4-7): odd counts leave
    a last single vector, 4100 rows a partial tile. Every vector within the
    tolerance of the oracle and of its own batch-1 call."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(40 + n_vec + t)
    out_dim, in_dim = 4100, 7168
    w = synth.matrix_host(rng, t, out_dim, in_dim)
    X = rng.standard_normal((n_vec, in_dim)).astype(np.float32)
    X[1] *= 1e3          # a different x exponent per vector
    wd = _dev(torch, w)
    got = ops.matvec_q(t, wd, _dev(torch, X), out_dim, in_dim).cpu().numpy()
    for v in range(n_vec):
        want = oracle.qlinear(t, w, out_dim, in_dim, X[v], nthreads=8)
        assert oracle.rel_err(got[v], want) <= TOL, v
        one = ops.matvec_q(t, wd, _dev(torch, np.ascontiguousarray(X[v])), out_dim, in_dim).cpu().numpy()
        assert oracle.rel_err(got[v], one) <= TOL, v


@pytest.mark.parametrize("rows", [2048, 7168, 16384])
@pytest.mark.parametrize("t", [Q.IQ1_S, Q.IQ2_XXS])
def test_config3_full_rows(torch_cuda, oracle, t, rows):
    """BASELINE configuration 3 at its full shapes, batch 1."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(rows + t)
    w = synth.matrix_host(rng, t, rows, 7168)
    x = rng.standard_normal(7168).astype(np.float32)
    want = oracle.qlinear(t, w, rows, 7168, x, nthreads=8)
    got = ops.matvec_q(t, _dev(torch, w), _dev(torch, x), rows, 7168).cpu().numpy()
    assert oracle.rel_err(got, want) <= TOL


@pytest.mark.parametrize("n_vec", [4, 16])
@pytest.mark.parametrize("rows", [2048, 7168, 16384])
@pytest.mark.parametrize("t", [Q.IQ1_S, Q.IQ2_XXS])
def test_config3_full_rows_batched(torch_cuda, oracle, t, rows, n_vec):
    """BASELINE configuration 3 at its full shapes for batches 4 and 16:
    every vector within 1e-4 of the oracle's qlinear of that vector."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(rows * 31 + t * 7 + n_vec)
    w = synth.matrix_host(rng, t, rows, 7168)
    X = rng.standard_normal((n_vec, 7168)).astype(np.float32)
    want = oracle.qlinear_batch(t, w, rows, 7168, X, nthreads=oracle.nproc())
    got = ops.matvec_q(t, _dev(torch, w), _dev(torch, X), rows, 7168).cpu().numpy()
    for v in range(n_vec):
        assert oracle.rel_err(got[v], want[v]) <= TOL, v


def test_config1_swiglu_slab(torch_cuda, oracle):
    """y = down(silu(gate x) * (up x)), Q2_K,
    2048x7168 / 7168x2048, x ~ N(0,1) seed 0."""
    from sepia_b200 import ops
    torch = torch_cuda
    rng = np.random.default_rng(0)
    x = rng.standard_normal(7168).astype(np.float32)
    g = synth.matrix_host(rng, Q.Q2_K, 2048, 7168)
    u = synth.matrix_host(rng, Q.Q2_K, 2048, 7168)
    d = synth.matrix_host(rng, Q.Q2_K, 7168, 2048)
    want = oracle.expert_swiglu(Q.Q2_K, g, Q.Q2_K, u, Q.Q2_K, d, 7168, 2048, x, nthreads=8)
    xd = _dev(torch, x)
    gv = ops.matvec_q(Q.Q2_K, _dev(torch, g), xd, 2048, 7168)
    uv = ops.matvec_q(Q.Q2_K, _dev(torch, u), xd, 2048, 7168)
    from sepia_b200.lib import load, ok
    h = torch.empty(2048, dtype=torch.float32, device="cuda")
    ok(load().sepia_cuda_silu_mul(gv.data_ptr(), uv.data_ptr(), h.data_ptr(), 2048, torch.cuda.current_stream().cuda_stream))
    y = ops.matvec_q(Q.Q2_K, _dev(torch, d), h, 7168, 2048).cpu().numpy()
    assert oracle.rel_err(y, want) <= TOL


@pytest.mark.parametrize("types", [(Q.Q2_K, Q.Q2_K, Q.Q2_K), (Q.IQ2_XS, Q.IQ2_XS, Q.IQ3_XXS)],
                         ids=["q2k", "iq2xs_iq3xxs"])
def test_expert_swiglu_entry(torch_cuda, oracle, types):
    """sepia_cuda_expert_swiglu (two engine launches) on BASELINE
    configuration 1's shapes, against the oracle's real_expert_ffn; run
    twice (the fixed one-slot selection is reused)."""
    from sepia_b200.lib import load, ok
    torch = torch_cuda
    tg, tu, td = types
    rng = np.random.default_rng(0)
    x = rng.standard_normal(7168).astype(np.float32)
    g = synth.matrix_host(rng, tg, 2048, 7168)
    u = synth.matrix_host(rng, tu, 2048, 7168)
    d = synth.matrix_host(rng, td, 7168, 2048)
    want = oracle.expert_swiglu(tg, g, tu, u, td, d, 7168, 2048, x, nthreads=8)
    gd, ud, dd, xd = _dev(torch, g), _dev(torch, u), _dev(torch, d), _dev(torch, x)
    h = torch.empty(2048, dtype=torch.float32, device="cuda")
    for _ in range(2):
        y = torch.full((7168,), float("nan"), dtype=torch.float32, device="cuda")
        ok(load().sepia_cuda_expert_swiglu(tg, gd.data_ptr(), tu, ud.data_ptr(), td, dd.data_ptr(), 7168, 2048,
                                           xd.data_ptr(), h.data_ptr(), y.data_ptr(),
                                           torch.cuda.current_stream().cuda_stream))
        assert oracle.rel_err(y.cpu().numpy(), want) <= TOL


def test_bad_arguments_rejected(torch_cuda):
    from sepia_b200.lib import load
    torch = torch_cuda
    L = load()
    w = torch.zeros(1024, dtype=torch.uint8, device="cuda")
    x = torch.zeros(300, dtype=torch.float32, device="cuda")
    y = torch.zeros(4, dtype=torch.float32, device="cuda")
    assert L.sepia_cuda_matvec_q(99, w.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 256, 1, None) == 0
    assert L.sepia_cuda_matvec_q(Q.Q4_K, w.data_ptr(), x.data_ptr(), y.data_ptr(), 4, 300, 1, None) == 0
    assert "block-aligned" in L.sepia_cuda_last_error().decode() or "unsupported" in L.sepia_cuda_last_error().decode()
    assert L.sepia_cuda_dequant(Q.Q2_K, w.data_ptr(), y.data_ptr(), 100, None) == 0
