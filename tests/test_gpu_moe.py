"""GPU: the device-resident MoE layer against the oracle's mlp_moe_forward
restatement (src/sepia.c:1377-1470, router src/sepia.c:1329-1375).

Router ids must match exactly; expert outputs within max relative error 1e-4.
Expert sharding (world > 1) must reproduce the world = 1 result bit for bit.
"""
import ctypes as C

import numpy as np
import pytest

from sepia_b200 import quants as Q
from sepia_b200.synth import MoeShape, hidden_state, moe_layer_host

pytestmark = pytest.mark.gpu
TOL = 1e-4

SHAPES = {
    "baseline_types_small": MoeShape(hidden=1024, ff=512, n_routed=64),
    "baseline_types_full_dims": MoeShape(hidden=7168, ff=2048, n_routed=12),
    "inkling_real_types": MoeShape(hidden=6144, ff=3072, n_routed=12, gate_type=Q.IQ2_XS, up_type=Q.IQ2_XS,
                                   down_type=Q.IQ3_XXS, sh_gate_type=Q.Q5_K, sh_up_type=Q.Q5_K,
                                   sh_down_type=Q.Q6_K),
    "iq4_down_q8_shared": MoeShape(hidden=2048, ff=1024, n_routed=16, gate_type=Q.IQ2_XS, up_type=Q.IQ2_XS,
                                   down_type=Q.IQ4_XS, sh_gate_type=Q.Q8_0, sh_up_type=Q.Q8_0,
                                   sh_down_type=Q.Q8_0),
    "no_shared_topk8": MoeShape(hidden=1024, ff=256, n_routed=32, n_shared=0, topk=8),
}


@pytest.fixture(scope="module")
def layers(lib):
    import torch
    from sepia_b200.moe import MoeLayerDevice
    out = {}
    for name, shape in SHAPES.items():
        H = moe_layer_host(shape, seed=5)
        out[name] = (H, MoeLayerDevice.from_host(H))
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("name", list(SHAPES))
def test_moe_layer_vs_oracle(layers, oracle, name):
    import torch
    H, D = layers[name]
    for seed in (1, 2, 3, 17, 64):
        x = hidden_state(seed, H.hidden)
        want, logits, idx, w = oracle.moe_layer(H, x, nthreads=8)
        xd = torch.from_numpy(x).cuda()
        out = torch.empty(H.hidden, dtype=torch.float32, device="cuda")
        D.forward(xd, out)
        torch.cuda.synchronize()
        assert np.array_equal(D.topk_idx.cpu().numpy(), idx), (name, seed)
        assert oracle.rel_err(D.logits.cpu().numpy(), logits) <= 1e-6
        assert oracle.rel_err(D.weights.cpu().numpy(), w) <= 1e-5
        assert oracle.rel_err(out.cpu().numpy(), want) <= TOL, (name, seed)


def test_router_bitexact_logits(layers, oracle):
    """fp64-accumulated router logits round to the same floats as dotf."""
    import torch
    H, D = layers["baseline_types_full_dims"]
    for seed in range(1, 9):
        x = hidden_state(seed, H.hidden)
        want = oracle.linear(H.router_w, x)
        D.forward(torch.from_numpy(x).cuda(), torch.empty(H.hidden, device="cuda"))
        torch.cuda.synchronize()
        got = D.logits.cpu().numpy()
        assert np.count_nonzero(got.view(np.uint32) != want.view(np.uint32)) <= 1


def test_topk_select_ties(lib, oracle):
    import torch
    from sepia_b200 import ops
    rng = np.random.default_rng(0)
    for trial in range(20):
        s = rng.integers(0, 5, size=256).astype(np.float32) / 4   # many exact ties
        want = oracle.topk_scores(s, 6)
        got = ops.topk_select(torch.from_numpy(s).cuda(), 6).cpu().numpy()
        assert np.array_equal(got, want)


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_expert_sharding_bit_identical(layers, world):
    """Each rank computes its own experts into slot terms; summing the slot
    buffers (what the NCCL all-reduce does) and combining reproduces the
    single-GPU output exactly. Ranks are emulated one after another on one GPU."""
    import torch
    from sepia_b200.lib import load, ok
    from sepia_b200.moe import MoeLayerDevice
    H, D1 = layers["baseline_types_small"]
    ranks = [MoeLayerDevice.from_host(H, rank=r, world=world) for r in range(world)]
    L = load()
    for seed in (4, 9, 33):
        x = torch.from_numpy(hidden_state(seed, H.hidden)).cuda()
        ref = torch.empty(H.hidden, device="cuda")
        D1.forward(x, ref)
        total = torch.zeros_like(ranks[0].slots)
        for R in ranks:
            st = torch.cuda.current_stream().cuda_stream
            ok(L.sepia_cuda_moe_router(C.byref(R.struct), x.data_ptr(), C.byref(R.ws), st))
            ok(L.sepia_cuda_moe_experts(C.byref(R.struct), x.data_ptr(), C.byref(R.ws), None, 1, st))
            total += R.slots
        R0 = ranks[0]
        R0.slots.copy_(total)
        out = torch.empty(H.hidden, device="cuda")
        ok(L.sepia_cuda_moe_combine(C.byref(R0.struct), C.byref(R0.ws), out.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int32), ref.view(torch.int32)), seed


def test_repeat_is_deterministic(layers):
    import torch
    H, D = layers["baseline_types_full_dims"]
    x = torch.from_numpy(hidden_state(7, H.hidden)).cuda()
    a = torch.empty(H.hidden, device="cuda")
    b = torch.empty(H.hidden, device="cuda")
    D.forward(x, a)
    D.forward(x, b)
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.mark.parametrize("n_routed,n_shared,dup", [(256, 2, False), (256, 2, True), (384, 2, True),
                                                    (1022, 2, False), (1024, 0, True)])
def test_router_selection_wide_and_ties(lib, oracle, n_routed, n_shared, dup):
    """Router ids and weights for expert counts on both sides of the one-warp
    selection's 256-entry register split, with exact score ties (duplicated
    router rows and biases: the lower index must win)."""
    import torch
    from sepia_b200.lib import ok
    from sepia_b200.moe import MoeLayerDevice
    shape = MoeShape(hidden=1024, ff=256, n_routed=n_routed, n_shared=n_shared, topk=6)
    rng = np.random.default_rng(n_routed)
    n_total = n_routed + n_shared
    w = (rng.standard_normal((n_total, shape.hidden), dtype=np.float32) * np.float32(0.02))
    bias = rng.uniform(-0.1, 0.1, size=n_routed).astype(np.float32)
    if dup:
        w[1:n_routed:2] = w[0:n_routed - 1:2]
        bias[1::2] = bias[0:n_routed - 1:2]
        bias[:] = np.round(bias * 8) / 8      # many equal biases across pairs too
    D = MoeLayerDevice.random(shape, seed=3)
    D.router_w.copy_(torch.from_numpy(w))
    D.router_bias.copy_(torch.from_numpy(bias))
    st = torch.cuda.current_stream().cuda_stream
    for seed in (1, 2, 5, 11):
        x = torch.from_numpy(hidden_state(seed, shape.hidden)).cuda()
        ok(lib.sepia_cuda_moe_router(C.byref(D.struct), x.data_ptr(), C.byref(D.ws), st))
        torch.cuda.synchronize()
        logits = D.logits.cpu().numpy()
        idx, wt = oracle.route_select(logits, bias, n_routed, n_shared, 6, shape.route_scale, shape.global_scale)
        assert np.array_equal(D.topk_idx.cpu().numpy(), idx), (seed, D.topk_idx.cpu().numpy(), idx)
        assert oracle.rel_err(D.weights.cpu().numpy(), wt) <= 1e-5, seed


def _device_layer_oracle(oracle, D, x, host_cache):
    """The oracle's mlp_moe_forward (src/sepia.c:1377-1470) for a layer whose
    expert store lives on the GPU: the router runs on the host copy of the
    f32 router, and only the selected experts' bytes are copied back."""
    s = D.shape
    if "router_w" not in host_cache:
        host_cache["router_w"] = D.router_w.cpu().numpy()
        host_cache["router_bias"] = D.router_bias.cpu().numpy()
        sg, su, sd = D.strides[3:]
        ng = Q.row_bytes(s.sh_gate_type, s.hidden) * s.ff
        nu = Q.row_bytes(s.sh_up_type, s.hidden) * s.ff
        nd = Q.row_bytes(s.sh_down_type, s.ff) * s.hidden
        host_cache["shared"] = [(D.sh_gate[k * sg:k * sg + ng].cpu().numpy(), D.sh_up[k * su:k * su + nu].cpu().numpy(),
                                 D.sh_down[k * sd:k * sd + nd].cpu().numpy()) for k in range(s.n_shared)]
    nt = oracle.nproc()
    logits = oracle.linear(host_cache["router_w"], x, nthreads=nt)
    idx, w = oracle.route_select(logits, host_cache["router_bias"], s.n_routed, s.n_shared, s.topk,
                                 s.route_scale, s.global_scale)
    out = np.zeros(s.hidden, np.float32)
    for j, e in enumerate(idx):
        g, u, d = D.expert_bytes_host(int(e))
        y = oracle.expert_swiglu(s.gate_type, g, s.up_type, u, s.down_type, d, s.hidden, s.ff, x, nthreads=nt)
        out += y * w[j]        # routed weight applied after down (src/sepia.c:1425)
    for k, (g, u, d) in enumerate(host_cache["shared"]):
        out += oracle.expert_swiglu(s.sh_gate_type, g, s.sh_up_type, u, s.sh_down_type, d, s.hidden, s.ff, x,
                                    w[s.topk + k], nthreads=nt)
    return out, logits, idx, w


def test_config2_full_layer_seeds_1_to_64(lib, oracle):
    """BASELINE configuration 2 at full size: 256 routed experts (Q2_K
    gate/up, Q3_K down), 2 shared Q4_K experts, the f32 [258 x 7168] router,
    hidden states of seeds 1-64. Router ids exact, output within 1e-4."""
    import torch
    from sepia_b200.moe import MoeLayerDevice
    from sepia_b200.synth import MoeShape as S
    shape = S()
    D = MoeLayerDevice.random(shape, seed=2)
    cache = {}
    out = torch.empty(shape.hidden, dtype=torch.float32, device="cuda")
    worst = 0.0
    for seed in range(1, 65):
        x = hidden_state(seed, shape.hidden)
        D.forward(torch.from_numpy(x).cuda(), out)
        torch.cuda.synchronize()
        want, logits, idx, w = _device_layer_oracle(oracle, D, x, cache)
        assert np.array_equal(D.topk_idx.cpu().numpy(), idx), seed
        assert oracle.rel_err(D.weights.cpu().numpy(), w) <= 1e-5, seed
        err = oracle.rel_err(out.cpu().numpy(), want)
        worst = max(worst, err)
        assert err <= TOL, (seed, err)
    del D
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", ["baseline_types_small", "baseline_types_full_dims"])
def test_fused_layer_matches_kernel_chain(layers, lib, name):
    """The single-launch layer (router, top-k, gate/up, down and combine in
    one persistent kernel) against the four-kernel chain on the same inputs:
    identical expert ids and weights, outputs within 1e-6 (the two paths sum
    the fp64 partials of a row in different groupings). Repeated calls and a
    CUDA-graph replay check that every launch leaves its counters zeroed."""
    import torch
    from sepia_b200.lib import ok
    H, D = layers[name]
    Ls, ws = C.byref(D.struct), C.byref(D.ws)
    assert lib.sepia_cuda_moe_fused_eligible(Ls, ws) == 1
    st = torch.cuda.current_stream().cuda_stream
    out_f = torch.empty(H.hidden, device="cuda")
    out_c = torch.empty(H.hidden, device="cuda")
    xin = torch.empty(H.hidden, device="cuda")
    g = None
    for rep, seed in enumerate((3, 9, 3, 40)):
        x = torch.from_numpy(hidden_state(seed, H.hidden)).cuda()
        ok(lib.sepia_cuda_moe_router(Ls, x.data_ptr(), ws, st))
        ok(lib.sepia_cuda_moe_experts(Ls, x.data_ptr(), ws, out_c.data_ptr(), 0, st))
        torch.cuda.synchronize()
        idx_c, w_c = D.topk_idx.clone(), D.weights.clone()
        if rep < 3:
            ok(lib.sepia_cuda_moe_layer_fused(Ls, x.data_ptr(), ws, out_f.data_ptr(), st))
        else:
            xin.copy_(x)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                ok(lib.sepia_cuda_moe_layer_fused(Ls, xin.data_ptr(), ws, out_f.data_ptr(),
                                                  torch.cuda.current_stream().cuda_stream))
            for _ in range(3):
                g.replay()
        torch.cuda.synchronize()
        assert lib.sepia_cuda_device_error(None) == 0
        assert torch.equal(D.topk_idx, idx_c), (rep, seed)
        assert torch.equal(D.weights, w_c), (rep, seed)
        a, b = out_f.cpu().numpy().astype(np.float64), out_c.cpu().numpy().astype(np.float64)
        den = np.maximum(np.abs(b), 1e-3 * np.abs(b).max())
        assert float(np.max(np.abs(a - b) / den)) <= 1e-6, (rep, seed)


def test_fused_not_taken_for_other_formats(layers, lib):
    """Layers whose experts are not in the tensor-core formats are not eligible."""
    H, D = layers["inkling_real_types"]
    assert lib.sepia_cuda_moe_fused_eligible(C.byref(D.struct), C.byref(D.ws)) == 0
