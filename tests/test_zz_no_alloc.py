"""GPU: the allocation-free banded attention entry point
(sepia_cuda_banded_attn_noalloc) against the workspace entry point
(sepia_cuda_banded_attn) on the same inputs, through the C ABI.

The file name sorts last so that pytest collects it after every other test:
it must pass both alone in a fresh process (the first call then performs the
per-device scratch address lookup) and after the rest of the suite."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-4

# (T, H, Hkv, Dh, rel_extent, q_pos_base, window, tau)
CASES = {
    "decode_config4_shape": (1, 64, 8, 128, 256, 3000, 0, 1.21),
    "prefill_window": (16, 8, 2, 64, 32, 100, 48, 1.0),
}
# partials of 256 * 64 * 130 * 8 = 17 MB per split: above the fixed scratch
OVERSIZED = (256, 64, 8, 128, 256, 0, 0, 1.0)


def _case(name):
    import torch
    T, H, Hkv, Dh, E, base, window, tau_v = OVERSIZED if name == "oversized" else CASES[name]
    rng = np.random.default_rng(len(name))
    kv_dim = Hkv * Dh
    cap = base + T
    pos = base + np.arange(T)
    lo = (np.maximum(0, pos - window + 1) if window else np.zeros(T)).astype(np.int64)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dict(
        q=d(rng.standard_normal(T * H * Dh).astype(np.float32)),
        k=d(rng.standard_normal(cap * kv_dim).astype(np.float32)).half(),
        v=d(rng.standard_normal(cap * kv_dim).astype(np.float32)).half(),
        rl=d((rng.standard_normal(T * H * E) * 0.5).astype(np.float32)),
        lo=d(lo), hi=d(pos.astype(np.int64)), tau=d(np.full(T, tau_v, np.float32)),
        T=T, H=H, Hkv=Hkv, Dh=Dh, E=E, base=base, kv_dim=kv_dim, max_kv=int((pos - lo).max()) + 1)


def _common(c, out):
    p = lambda t: C.c_void_p(t.data_ptr())
    return [1, p(c["q"]), p(c["k"]), p(c["v"]), p(c["rl"]), p(out), p(c["lo"]), p(c["hi"]), p(c["tau"]),
            c["T"], c["H"], c["Hkv"], c["Dh"], c["E"], c["base"], c["kv_dim"], 1.0 / c["Dh"], c["max_kv"]]


def _with_workspace(lib, c):
    import torch
    out = torch.empty(c["T"] * c["H"] * c["Dh"], dtype=torch.float32, device="cuda")
    wsb = lib.sepia_cuda_banded_attn_ws_bytes(c["T"], c["H"], c["Hkv"], c["Dh"], c["max_kv"])
    ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
    assert lib.sepia_cuda_banded_attn(*_common(c, out), C.c_void_p(ws.data_ptr()), wsb, None) == 1
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _no_alloc(lib, c):
    import torch
    out = torch.full((c["T"] * c["H"] * c["Dh"],), float("nan"), dtype=torch.float32, device="cuda")
    assert lib.sepia_cuda_banded_attn_noalloc(*_common(c, out), None) == 1, lib.sepia_cuda_last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _rel_err(got, want):
    scale = float(np.max(np.abs(want)))
    den = np.maximum(np.abs(want).astype(np.float64), max(1e-6, 1e-3 * scale))
    return float(np.max(np.abs(got.astype(np.float64) - want) / den))


def _oracle_want(oracle, c):
    """The CPU restatement of attn_forward_chunk's inner loop on the same inputs."""
    h = lambda t: t.float().cpu().numpy() if t.dtype == __import__("torch").float16 else t.cpu().numpy()
    return oracle.banded_attn(h(c["q"]), h(c["k"]), h(c["v"]), h(c["rl"]), h(c["lo"]), h(c["hi"]), h(c["tau"]),
                              c["T"], c["H"], c["Hkv"], c["Dh"], c["E"], c["base"], c["kv_dim"], 1.0 / c["Dh"],
                              nthreads=oracle.nproc())


@pytest.mark.parametrize("name", list(CASES))
def test_no_alloc_matches_workspace_entry(lib, oracle, name):
    """Two calls of this shape with a call of the other shape and other
    inputs between them: the scratch array keeps the last call's partials,
    so stale contents would show up in the second result. Both must equal
    the workspace entry point bit for bit (same kernels, same split count)
    and lie within 1e-4 of the CPU oracle."""
    other = [n for n in CASES if n != name][0]
    c, c_other = _case(name), _case(other)
    want = _with_workspace(lib, c)
    first = _no_alloc(lib, c)
    between = _no_alloc(lib, c_other)
    second = _no_alloc(lib, c)
    assert np.array_equal(between.view(np.uint32), _with_workspace(lib, c_other).view(np.uint32))
    assert np.array_equal(first.view(np.uint32), want.view(np.uint32))
    assert np.array_equal(second.view(np.uint32), want.view(np.uint32))
    assert _rel_err(first, _oracle_want(oracle, c)) <= TOL


def test_no_alloc_rejects_oversized_shape(lib):
    import torch
    cap = lib.sepia_cuda_banded_attn_noalloc_max_bytes()
    assert cap == 8 << 20
    c = _case("oversized")      # full-size buffers, so even a wrong accept stays in bounds
    assert lib.sepia_cuda_banded_attn_ws_bytes(c["T"], c["H"], c["Hkv"], c["Dh"], c["max_kv"]) > cap
    out = torch.empty(c["T"] * c["H"] * c["Dh"], dtype=torch.float32, device="cuda")
    assert lib.sepia_cuda_banded_attn_noalloc(*_common(c, out), None) == 0
    msg = lib.sepia_cuda_last_error()
    msg = msg.decode() if isinstance(msg, bytes) else str(msg)
    assert "scratch" in msg
