"""GPU: the reference-shaped ABI (include/sepia_gpu.h) through ctypes --
buffer semantics, batching rules, error returns, and each f32 op against the
oracle. Mirrors the reference's own --gpu-selftest (src/sepia.c:4469-4548)."""
import ctypes as C
import mmap

import numpy as np
import pytest

from sepia_b200 import quants as Q
from sepia_b200 import synth

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def G(lib):
    assert lib.sepia_gpu_available() == 1
    assert lib.sepia_gpu_init(b"metal") == 1
    assert b"B200" in lib.sepia_gpu_device_name() or lib.sepia_gpu_device_name()
    return lib


def put(G, a):
    a = np.ascontiguousarray(a)
    b = G.sepia_gpu_alloc(max(a.nbytes, 4), 0)
    assert b
    C.memmove(G.sepia_gpu_host_ptr(b), a.ctypes.data, a.nbytes)
    return b


def get(G, b, n, dtype=np.float32):
    out = np.empty(n, dtype)
    C.memmove(out.ctypes.data, G.sepia_gpu_host_ptr(b), out.nbytes)
    return out


def test_selftest_semantics(G):
    page = mmap.PAGESIZE
    m = mmap.mmap(-1, 3 * page)
    arr = np.frombuffer(m, dtype=np.float32)
    arr[:] = np.arange(arr.size, dtype=np.float32)
    base = C.addressof(C.c_char.from_buffer(m))
    b = G.sepia_gpu_wrap_mmap(base, 3 * page)
    assert b
    assert G.sepia_gpu_host_ptr(b) == base
    assert G.sepia_gpu_selftest_touch(b, page // 4) == 1
    assert np.array_equal(arr, np.arange(arr.size, dtype=np.float32))
    assert not G.sepia_gpu_wrap_mmap(base + 1, page)        # misaligned -> NULL
    G.sepia_gpu_free(b)
    del arr
    m.close()
    s = G.sepia_gpu_alloc(page, 0)
    p = G.sepia_gpu_alloc(page, 1)
    assert G.sepia_gpu_host_ptr(s) and not G.sepia_gpu_host_ptr(p)
    assert G.sepia_gpu_gpu_addr(p) != 0
    G.sepia_gpu_free(s)
    G.sepia_gpu_free(p)
    G.sepia_gpu_free(None)


def test_batching_rules(G):
    x = put(G, np.ones(16, np.float32))
    y = put(G, np.zeros(16, np.float32))
    assert G.sepia_gpu_add(x, x, y, 16) == 0            # no batch open
    assert G.sepia_gpu_end() == 0
    assert G.sepia_gpu_flush() == 0
    assert G.sepia_gpu_begin() == 1
    assert G.sepia_gpu_begin() == 0                      # already open
    assert G.sepia_gpu_add(x, x, y, 16) == 1
    assert G.sepia_gpu_flush() == 1
    assert G.sepia_gpu_scale(3.0, y, y, 16) == 1
    assert G.sepia_gpu_add(x, x, y, 17) == 0             # out of bounds -> rejected
    assert G.sepia_gpu_end() == 1
    assert np.array_equal(get(G, y, 16), np.full(16, 6.0, np.float32))
    for b in (x, y):
        G.sepia_gpu_free(b)


def test_f32_ops_vs_oracle(G, oracle):
    rng = np.random.default_rng(11)
    rows, n = 3, 1000
    x = rng.standard_normal(rows * n).astype(np.float32)
    w = rng.standard_normal(n).astype(np.float32)
    W = (rng.standard_normal((258, 1024)) * 0.02).astype(np.float32)
    v = rng.standard_normal(1024).astype(np.float32)
    g = rng.standard_normal(777).astype(np.float32)
    u = rng.standard_normal(777).astype(np.float32)
    bx, bw, by = put(G, x), put(G, w), put(G, np.zeros(rows * n, np.float32))
    bW, bv, bo = put(G, W), put(G, v), put(G, np.zeros(258, np.float32))
    bg, bu, bz = put(G, g), put(G, u), put(G, np.zeros(777, np.float32))
    bs = put(G, np.zeros(rows * n, np.float32))
    assert G.sepia_gpu_begin() == 1
    assert G.sepia_gpu_rmsnorm(bw, bx, by, rows, n, np.float32(1e-5)) == 1
    assert G.sepia_gpu_matvec(bW, bv, bo, 258, 1024) == 1
    assert G.sepia_gpu_silu_mul(bg, bu, bz, 777) == 1
    assert G.sepia_gpu_softmax(bx, bs, rows, n) == 1
    assert G.sepia_gpu_end() == 1
    L = oracle.lib()
    want = np.empty(rows * n, np.float32)
    for r in range(rows):
        part = np.empty(n, np.float32)
        L.or_rmsnorm(np.ascontiguousarray(x[r * n:(r + 1) * n]), w, n, np.float32(1e-5), part)
        want[r * n:(r + 1) * n] = part
    assert oracle.rel_err(get(G, by, rows * n), want) <= 1e-6
    assert oracle.rel_err(get(G, bo, 258), oracle.linear(W, v)) <= 1e-6
    z = np.empty(777, np.float32)
    L.or_silu_mul(g, u, z, 777)
    assert oracle.rel_err(get(G, bz, 777), z) <= 1e-6
    sm = np.empty(rows * n, np.float32)
    L.or_softmax_rows(x, sm, rows, n)
    assert oracle.rel_err(get(G, bs, rows * n), sm) <= 1e-6


def test_sconv_and_hist_roll(G, oracle):
    rng = np.random.default_rng(5)
    L = oracle.lib()
    for (Cc, K, T) in [(64, 4, 1), (64, 4, 2), (128, 4, 7), (32, 16, 3)]:
        w = (rng.standard_normal(Cc * K) * 0.1).astype(np.float32)
        hist = rng.standard_normal((K - 1) * Cc).astype(np.float32)
        inp = rng.standard_normal(T * Cc).astype(np.float32)
        bw, bh, bi, bo = put(G, w), put(G, hist), put(G, inp), put(G, np.zeros(T * Cc, np.float32))
        assert G.sepia_gpu_begin() == 1
        assert G.sepia_gpu_sconv(bw, bh, bi, bo, Cc, K, T) == 1
        assert G.sepia_gpu_sconv_hist_roll(bh, bi, Cc, K, T) == 1
        assert G.sepia_gpu_end() == 1
        want = np.empty(T * Cc, np.float32)
        h2 = hist.copy()
        L.or_sconv_apply(w, Cc, K, h2, inp, T, want)
        assert oracle.rel_err(get(G, bo, T * Cc), want) <= 1e-6
        assert np.array_equal(get(G, bh, (K - 1) * Cc), h2)          # pure data movement: bitwise
    assert G.sepia_gpu_begin() == 1
    assert G.sepia_gpu_sconv_hist_roll(bh, bi, 4, 17, 1) == 0        # K-1 > 15 rejected
    assert G.sepia_gpu_end() == 1


def test_matvec_q_dequant_rows_and_offsets(G, oracle):
    rng = np.random.default_rng(9)
    for t in Q.QUANT_TYPES:
        out_dim, in_dim = 8, 512
        w = synth.matrix_host(rng, t, out_dim, in_dim)
        pad = np.zeros(48, np.uint8)
        blob = np.concatenate([pad, w])
        x = rng.standard_normal(in_dim).astype(np.float32)
        bw, bx = put(G, blob), put(G, x)
        by, bd = put(G, np.zeros(out_dim, np.float32)), put(G, np.zeros(out_dim * in_dim, np.float32))
        assert G.sepia_gpu_begin() == 1
        assert G.sepia_gpu_matvec_q(t, bw, 48, bx, by, out_dim, in_dim) == 1
        assert G.sepia_gpu_dequant_rows(t, bw, 48, bd, out_dim * in_dim) == 1
        assert G.sepia_gpu_end() == 1
        assert oracle.rel_err(get(G, by, out_dim), oracle.qlinear(t, w, out_dim, in_dim, x)) <= 1e-4
        want = oracle.dequantize(t, w, out_dim * in_dim)
        assert np.array_equal(get(G, bd, out_dim * in_dim).view(np.uint32), want.view(np.uint32))
        for b in (bw, bx, by, bd):
            G.sepia_gpu_free(b)


def test_copy_and_moe_extension(G, oracle):
    from sepia_b200.synth import MoeShape, hidden_state, moe_layer_host
    from sepia_b200.lib import SepiaGpuMoeDesc
    shape = MoeShape(hidden=1024, ff=512, n_routed=16)
    H = moe_layer_host(shape, seed=3)
    sg, su, sd, ssg, ssu, ssd = shape.strides()
    experts = np.concatenate([H.gate, H.up, H.down])
    shared = np.concatenate([H.sh_gate, H.sh_up, H.sh_down])
    be, bsh = put(G, experts), put(G, shared)
    brw, brb = put(G, H.router_w), put(G, H.router_bias)
    d = SepiaGpuMoeDesc()
    d.hidden, d.ff, d.n_routed, d.n_shared, d.topk = 1024, 512, 16, 2, 6
    d.route_scale, d.global_scale = 8.0, 1.0
    d.router_w, d.router_bias = brw, brb
    d.gate_type, d.up_type, d.down_type = shape.gate_type, shape.up_type, shape.down_type
    d.experts, d.gate_off, d.up_off, d.down_off = be, 0, H.gate.size, H.gate.size + H.up.size
    d.gate_stride, d.up_stride, d.down_stride = sg, su, sd
    d.sh_gate_type, d.sh_up_type, d.sh_down_type = shape.sh_gate_type, shape.sh_up_type, shape.sh_down_type
    d.shared, d.sh_gate_off, d.sh_up_off, d.sh_down_off = bsh, 0, H.sh_gate.size, H.sh_gate.size + H.sh_up.size
    d.sh_gate_stride, d.sh_up_stride, d.sh_down_stride = ssg, ssu, ssd
    x = hidden_state(12, 1024)
    bx, bo = put(G, x), put(G, np.zeros(1024, np.float32))
    bi, bwt = put(G, np.zeros(6, np.int32)), put(G, np.zeros(8, np.float32))
    bc = put(G, np.zeros(1024, np.float32))
    assert G.sepia_gpu_begin() == 1
    assert G.sepia_gpu_moe_layer(C.byref(d), bx, bo, bi, bwt) == 1
    assert G.sepia_gpu_copy(bo, 0, bc, 0, 1024) == 1
    assert G.sepia_gpu_end() == 1
    want, logits, idx, w = oracle.moe_layer(H, x, nthreads=4)
    assert np.array_equal(get(G, bi, 6, np.int32), idx)
    assert oracle.rel_err(get(G, bo, 1024), want) <= 1e-4
    assert np.array_equal(get(G, bc, 1024), get(G, bo, 1024))


def test_bounded_wait_timeout_reports_and_context_survives(lib):
    """Failure detection without a GPU fault: the engine's producer
    announces more bytes than it copies, every waiting role gives up after a
    short bound (2e6 cycles, ~1 ms) and records error 1; the host reads it
    through sepia_cuda_device_error and through sepia_gpu_end (which must
    return 0); afterwards the same call without the hook computes normally."""
    import torch
    from sepia_b200 import ops
    rng = np.random.default_rng(11)
    t, out_dim, in_dim = Q.Q2_K, 64, 2048
    w = torch.from_numpy(synth.matrix_host(rng, t, out_dim, in_dim)).cuda()
    x = torch.from_numpy(rng.standard_normal(in_dim).astype(np.float32)).cuda()
    y = torch.zeros(out_dim, dtype=torch.float32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.sepia_cuda_device_error(st) == 0
    assert lib.sepia_cuda_test_engine_timeout(t, w.data_ptr(), x.data_ptr(), y.data_ptr(), out_dim, in_dim,
                                              2_000_000, st) == 1
    assert lib.sepia_cuda_device_error(st) == 1
    assert lib.sepia_cuda_device_error(st) == 0          # read-and-clear
    # through the reference-shaped batch API: end() reports the failure
    assert lib.sepia_gpu_init(b"metal") == 1
    assert lib.sepia_gpu_begin() == 1
    assert lib.sepia_cuda_test_engine_timeout(t, w.data_ptr(), x.data_ptr(), y.data_ptr(), out_dim, in_dim,
                                              2_000_000, lib.sepia_cuda_lib_stream()) == 1
    assert lib.sepia_gpu_end() == 0
    assert b"device error" in lib.sepia_cuda_last_error()
    # the context still works
    good = ops.matvec_q(t, w, x, out_dim, in_dim)
    torch.cuda.synchronize()
    assert lib.sepia_cuda_device_error(st) == 0
    assert torch.isfinite(good).all()
