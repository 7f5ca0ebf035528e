#!/usr/bin/env python3
"""Headline benchmark: BASELINE configuration 2 -- one MoE layer of the
Inkling shape decoding one token (router f32 [258 x 7168] + sigmoid top-6 of
256 routed experts with Q2_K gate/up and Q3_K down, ff 2048, + 2 shared Q4_K
experts), weights resident in HBM, experts sharded over the GPUs.

A step is one token through one layer. Steps rotate over --layers distinct
layer instances (default 4, 4 x 152.6 MB touched per rotation > 126 MB L2),
so weights are never L2-resident. Each instance is replayed as one CUDA
graph holding its own resident hidden state (instance l: seed l+1), so each
instance selects the same 6 experts on every replay; the eager and e2e paths
rotate over hidden states of seeds 1..64.

value  = whole-job quantized-matvec HBM throughput: algorithmic bytes of
         the steps (152.6 MB/token: router + 6 routed + 2 shared experts +
         activations) / device time (max over ranks).
e2e    = the same through the reference-facing C ABI (include/sepia_gpu.h:
         sepia_gpu_begin / sepia_gpu_moe_layer / sepia_gpu_end) with host
         buffers: x uploaded and the layer output read back every step.
Run:   python bench.py [--gpus N --steps K --warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import re
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Q-matvec HBM GB/s (% of 8 TB/s); synthetic Inkling-shape decode tok/s"
PEAKS = ROOT / "MEASURED_PEAKS.json"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="sepia", choices=["sepia", "reference"])
    ap.add_argument("--layers", type=int, default=4, help="distinct layer instances rotated per step")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="eager launches instead of one CUDA graph per layer")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--parity", action="store_true", help="check one step against the CPU oracle")
    ap.add_argument("--only", default="", help="kernels workload: run only the lines whose name contains this")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-5 decode measurement")
    ap.add_argument("--no-kernels", action="store_true", help="skip the config-1/3/4 kernel lines in the default run")
    ap.add_argument("--decode-layers", type=int, default=0, help="config-5 depth (default 24 at N=1, 66 at N>1)")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--gen", type=int, default=256)
    ap.add_argument("--workload", default="moe_layer", choices=["moe_layer", "kernels", "decode"],
                    help="moe_layer: the headline line (config 2); kernels: one line per BASELINE config-1/3/4 "
                         "kernel (device time, 1 GPU)")
    return ap.parse_args()


def peak_hbm():
    try:
        d = json.loads(PEAKS.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------- clocks
class Clocks:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.p = None
        self.index = index
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if not self.p:
            return None
        time.sleep(0.25)
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            return None
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [s.strip() for s in line.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------- CPU
def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuLayer:
    """Host copy of one config-2 layer for the CPU baseline: the f32 router,
    6 distinct routed experts (the ones a token selects) and 2 shared."""

    def __init__(self, shape, seed=11):
        import numpy as np
        from sepia_b200 import synth
        s = shape
        rng = np.random.default_rng(seed)
        self.s = s
        self.routed = [tuple(synth.matrix_host(rng, t, r, c) for t, r, c in [
            (s.gate_type, s.ff, s.hidden), (s.up_type, s.ff, s.hidden), (s.down_type, s.hidden, s.ff)])
            for _ in range(s.topk)]
        self.shared = [tuple(synth.matrix_host(rng, t, r, c) for t, r, c in [
            (s.sh_gate_type, s.ff, s.hidden), (s.sh_up_type, s.ff, s.hidden), (s.sh_down_type, s.hidden, s.ff)])
            for _ in range(s.n_shared)]
        self.rw = (rng.standard_normal((s.n_routed + s.n_shared, s.hidden)) * 0.02).astype(np.float32)

    def token(self, x, n):
        """Router matvec + 6 routed + 2 shared SwiGLU experts, n threads (the
        oracle port of the reference's qlinear loop: the reference itself has
        no Q2_K/Q3_K)."""
        from oracle import oracle as O
        s = self.s
        O.linear(self.rw, x, nthreads=n)
        for g, u, d in self.routed:
            O.expert_swiglu(s.gate_type, g, s.up_type, u, s.down_type, d, s.hidden, s.ff, x, nthreads=n)
        for g, u, d in self.shared:
            O.expert_swiglu(s.sh_gate_type, g, s.sh_up_type, u, s.sh_down_type, d, s.hidden, s.ff, x, 0.5,
                            nthreads=n)


def cpu_token_seconds(shape, budget_s=10.0):
    """Time the CPU baseline on tokens of the layer, all host threads and
    then one thread (the reference's own loop is single-threaded). Returns
    (seconds per token at n threads, n, sample description, seconds per
    token at 1 thread)."""
    from oracle import oracle as O
    from sepia_b200 import synth
    O.build()
    n = O.nproc()
    C_ = CpuLayer(shape)

    def timed(threads, budget, max_reps):
        reps, t_tot = 0, 0.0
        while True:
            x = synth.hidden_state(1 + reps % 64, shape.hidden)
            t0 = time.perf_counter()
            C_.token(x, threads)
            t_tot += time.perf_counter() - t0
            reps += 1
            if t_tot > budget or reps >= max_reps:
                return t_tot / reps, reps
    sec_n, reps_n = timed(n, budget_s, 50)
    sec_1, reps_1 = timed(1, budget_s, 3)
    return (sec_n, n, f"{reps_n} token(s) of config 2 (router + 6 distinct routed + 2 shared SwiGLU) on {n} "
                      f"threads; {reps_1} token(s) on 1 thread", sec_1)


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from sepia_b200.synth import MoeShape
    from oracle import oracle as O
    from sepia_b200 import synth
    shape = MoeShape()
    O.build()
    n = O.nproc()
    s = shape
    C_ = CpuLayer(shape)

    def step(i):
        C_.token(synth.hidden_state(1 + i % 64, s.hidden), n)

    for i in range(args.warmup):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = time.perf_counter() - t0
    gbs = args.steps * shape.token_bytes() / dt / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (BASELINE config 2 distributions)",
            "config": {"workload": "config2_moe_layer_decode_1tok", "hidden": 7168, "ff": 2048, "experts": 256,
                       "topk": 6, "shared": 2, "types": "Q2_K gate/up, Q3_K down, Q4_K shared"},
            "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": n, "kind": "port",
                             "cpu_model": cpu_model(),
                             "sample": f"{args.steps} tokens of config 2 (6 distinct routed experts) on {n} threads "
                                       "(oracle port of the reference qlinear loop; the reference lacks Q2_K/Q3_K)"},
            "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "layer_steps_per_s": round(args.steps / dt, 3)}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------- traffic
def committed_traffic():
    """dram bytes per launch of k_gateup from the committed ncu summary."""
    p = ROOT / "profiles" / "k_gateup_moe_layer.md"
    try:
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
        return float(m.group(1)) if m else None
    except Exception:
        return None


# ------------------------------------------------------------------ decode
def decode_measure(args, world, rank, group):
    """a random-init Inkling-shape model generated
    in HBM (24-layer truncation on one GPU, all 66 layers when experts are
    sharded), a 512-token prefill of random ids (seed 7), then 256 greedy
    decode steps replayed from one CUDA graph per step. Returns a dict (rank
    0) with decode tok/s, prefill tok/s and the decode HBM roofline."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from sepia_b200 import container as CT
    from sepia_b200.model import DeviceModel
    n_layers = args.decode_layers or (24 if world == 1 else 66)
    tc = CT.config5_text_config(n_layers)
    cfg = CT.ModelConfig.from_text_config(tc)
    types = CT.ModelTypes()
    t0 = time.perf_counter()
    m = DeviceModel.synthetic(cfg, types, seed=7, max_positions=args.prompt + args.gen + 8, rank=rank, world=world)
    m.connect(group)
    build_s = time.perf_counter() - t0
    prompt = np.random.default_rng(7).integers(0, cfg.vocab_size, args.prompt).astype(np.int32)
    ids = torch.as_tensor(prompt, device="cuda")
    out = torch.empty(args.gen, dtype=torch.int32, device="cuda")
    # warm-up: a short sequence (sets kernel attributes, captures the graph)
    m.reset()
    m.prefill(ids[:8], True)
    m.decode(out, 4)
    torch.cuda.synchronize()
    m.reset()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    if world > 1:
        dist.barrier()
    clk = Clocks(int(os.environ.get("LOCAL_RANK", "0"))) if rank == 0 else None
    torch.cuda.synchronize()
    e0.record()
    m.prefill(ids, True)
    e1.record()
    m.decode(out, args.gen)
    e2.record()
    torch.cuda.synchronize()
    clocks = clk.stop() if clk else None
    pre_ms, dec_ms = e0.elapsed_time(e1), e1.elapsed_time(e2)
    if world > 1:
        t = torch.tensor([pre_ms, dec_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        pre_ms, dec_ms = float(t[0]), float(t[1])
    tb = CT.token_bytes(cfg, types, args.prompt + args.gen // 2)
    peak, kind = peak_hbm()
    dec_tok_s = args.gen / (dec_ms / 1e3)
    gbs = tb["total"] * dec_tok_s / 1e9
    res = {"metric": "synthetic Inkling-shape decode tok/s", "value": round(dec_tok_s, 2), "unit": "tok/s",
           "prefill_tok_s": round(args.prompt / (pre_ms / 1e3), 2), "ms_per_token": round(dec_ms / args.gen, 4),
           "layers": n_layers, "prompt": args.prompt, "generated": args.gen, "n_gpus": world,
           "bytes_per_token": tb, "hbm_gbs": round(gbs, 1), "frac_of_measured_peak": round(gbs / peak, 4),
           "peak_kind": kind, "weights_gb_per_gpu": round(m.weight_bytes() / 1e9, 2), "build_s": round(build_s, 1),
           "first_ids": out[:8].cpu().tolist(), "graph": "one CUDA graph per decode step",
           "clocks": clocks}
    del m
    torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------- main
def kernel_lines(args):
    """Device-timed bandwidth of the other BASELINE kernels on one GPU:
    config 1 (Q2_K SwiGLU slab: three matvecs + silu_mul), config 3 (IQ1_S /
    IQ2_XXS matvec, rows 2048/7168/16384 x 7168, batch 1/4/16), config 4
    (banded attention decode, H=64 Hkv=8 Dh=128 fp16 K/V, global at 32768 and
    window 4096). Weights rotate through buffers larger than L2."""
    import torch
    from sepia_b200 import quants as Q, synth
    from sepia_b200.lib import load, ok
    L = load()
    peak, kind = peak_hbm()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)

    def timeit(fn, n):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        torch.cuda._sleep(50_000_000)
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        for i in range(n):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n * 1e-3

    recs = []

    def emit(name, nbytes, sec, extra):
        gbs = nbytes / sec / 1e9
        rec = {"metric": "kernel HBM GB/s", "kernel": name, "value": round(gbs, 1), "unit": "GB/s",
               "us": round(sec * 1e6, 2), "bytes": nbytes, "frac_of_measured_peak": round(gbs / peak, 4),
               "peak_kind": kind, "data": "synthetic", **extra}
        recs.append(rec)
        if args.workload == "kernels":
            print(json.dumps(rec), flush=True)

    def mats(t, rows, cols):
        nb = Q.row_bytes(t, cols) * rows
        return [synth.blocks_device(gen, t, rows * cols // Q.block_elems(t)) for _ in range(max(2, int(800e6 // nb)))]

    def want(name):
        return args.only in name

    if want("config1_q2k_swiglu_slab"):
        g, u, d = mats(Q.Q2_K, 2048, 7168), mats(Q.Q2_K, 2048, 7168), mats(Q.Q2_K, 7168, 2048)
        x = torch.randn(7168, device="cuda")
        ga, ua, y = torch.empty(2048, device="cuda"), torch.empty(2048, device="cuda"), torch.empty(7168, device="cuda")
        h = torch.empty(2048, device="cuda")

        def slab(i):
            k = i % len(g)
            ok(L.sepia_cuda_expert_swiglu(Q.Q2_K, g[k].data_ptr(), Q.Q2_K, u[k].data_ptr(), Q.Q2_K, d[k].data_ptr(),
                                          7168, 2048, x.data_ptr(), h.data_ptr(), y.data_ptr(), None))
        emit("config1_q2k_swiglu_slab", 14516224, timeit(slab, 100), {"launches": 2, "entry": "sepia_cuda_expert_swiglu"})
        del g, u, d
    for t, name in ((Q.IQ1_S, "iq1_s"), (Q.IQ2_XXS, "iq2_xxs")):
        for rows in (2048, 7168, 16384):
            if not any(want(f"config3_{name}_{rows}x7168_b{b}") for b in (1, 4, 16)):
                continue
            ws = mats(t, rows, 7168)
            for b in (1, 4, 16):
                if not want(f"config3_{name}_{rows}x7168_b{b}"):
                    continue
                xb = torch.randn(b, 7168, device="cuda")
                yb = torch.empty(b, rows, device="cuda")
                fn = lambda i: ok(L.sepia_cuda_matvec_q(t, ws[i % len(ws)].data_ptr(), xb.data_ptr(), yb.data_ptr(),
                                                        rows, 7168, b, None))
                nbytes = Q.row_bytes(t, 7168) * rows + 4 * b * (7168 + rows)
                emit(f"config3_{name}_{rows}x7168_b{b}", nbytes, timeit(fn, 50), {"rows": rows, "batch": b})
            del ws
    for ctx, window in ((32768, 0), (4096, 4096)):
        if not want(f"config4_attn_ctx{ctx}_{'global' if not window else 'window'}"):
            continue
        H, Hkv, Dh, E = 64, 8, 128, 256
        kvd = Hkv * Dh
        # K/V sets rotated per call: more than L2 (126 MB) in all
        nset = max(2, -(-300_000_000 // (ctx * kvd * 2 * 2)))
        ks = [torch.randn(ctx, kvd, device="cuda").half() for _ in range(nset)]
        vs = [torch.randn(ctx, kvd, device="cuda").half() for _ in range(nset)]
        q = torch.randn(H * Dh, device="cuda")
        rl = torch.randn(H * E, device="cuda") * 0.02
        hi = torch.tensor([ctx - 1], dtype=torch.int64, device="cuda")
        lo = torch.tensor([max(0, ctx - window) if window else 0], dtype=torch.int64, device="cuda")
        tau = torch.ones(1, device="cuda")
        out = torch.empty(H * Dh, device="cuda")
        max_kv = ctx - int(lo.item())
        wsb = L.sepia_cuda_banded_attn_ws_bytes(1, H, Hkv, Dh, max_kv)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")
        fn = lambda i: ok(L.sepia_cuda_banded_attn(1, q.data_ptr(), ks[i % nset].data_ptr(), vs[i % nset].data_ptr(),
                                                   rl.data_ptr(),
                                                   out.data_ptr(), lo.data_ptr(), hi.data_ptr(), tau.data_ptr(), 1, H,
                                                   Hkv, Dh, E, ctx - 1, kvd, 1.0 / Dh, max_kv, ws.data_ptr(), wsb,
                                                   None))
        nbytes = ctx * kvd * 2 * 2 + 4 * (H * Dh * 2 + H * E)
        emit(f"config4_attn_ctx{ctx}_{'global' if not window else 'window'}", nbytes, timeit(fn, 50),
             {"ctx": ctx, "kv_sets": nset, "l2": "K/V sets rotated per call, more than L2 in all"})
        del ks, vs, ws
    if want("moe_layer_real_types"):
        # the real Inkling expert formats: IQ2_XS gate/up, IQ3_XXS down
        # (routed), Q4_K shared experts; BASELINE config-2 geometry
        from sepia_b200.moe import MoeLayerDevice
        from sepia_b200.synth import MoeShape, hidden_state
        shape = MoeShape(gate_type=Q.IQ2_XS, up_type=Q.IQ2_XS, down_type=Q.IQ3_XXS)
        lays = [MoeLayerDevice.random(shape, seed=300 + i) for i in range(4)]
        X = torch.stack([torch.from_numpy(hidden_state(s, shape.hidden)) for s in range(1, 65)]).cuda()
        y = torch.empty(shape.hidden, device="cuda")
        st = torch.cuda.current_stream().cuda_stream

        def layer(i):
            D = lays[i % len(lays)]
            ok(L.sepia_cuda_moe_layer(C.byref(D.struct), X[i % 64].data_ptr(), C.byref(D.ws), y.data_ptr(), st))
        emit("moe_layer_real_types", shape.token_bytes(), timeit(layer, 100),
             {"types": "IQ2_XS gate/up, IQ3_XXS down, Q4_K shared, f32 router", "layer_instances": len(lays)})
        del lays
    return recs


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "kernels":
        kernel_lines(args)
        return
    import torch
    import torch.distributed as dist
    from sepia_b200 import lib as LIB
    from sepia_b200.moe import MoeLayerDevice
    from sepia_b200.synth import MoeShape, hidden_state

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    L = LIB.load()
    if args.workload == "decode":
        res = decode_measure(args, world, rank, group)
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    shape = MoeShape()
    layers = [MoeLayerDevice.random(shape, seed=100 + l, rank=rank, world=world) for l in range(args.layers)]
    if world > 1:
        # one NVLink slot exchange per rank, shared by the layer instances
        from sepia_b200.moe import Exchange
        xchg = Exchange(shape.topk + shape.n_shared, shape.hidden, rank, world)
        xchg.connect(group)
        for D in layers:
            D.exchange = xchg
    X = torch.stack([torch.from_numpy(hidden_state(s, shape.hidden)) for s in range(1, 65)]).cuda()
    out = torch.empty(shape.hidden, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    def step(i):
        layers[i % len(layers)].forward(X[i % 64], out, group=group)

    # Decode runs a layer as one CUDA graph (router, gate/up, down, combine
    # -- or, sharded, the NVLink slot exchange -- replayed without host
    # launch gaps). One graph per layer instance, each with its own resident
    # input.
    graphs = []
    if not args.no_graph:
        xin = X[:len(layers)].clone()
        outs = torch.empty(len(layers), shape.hidden, dtype=torch.float32, device="cuda")
        for l, D in enumerate(layers):      # warm: kernel attributes set before capture
            D.forward(xin[l], outs[l])
        torch.cuda.synchronize()
        for l, D in enumerate(layers):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                D.forward(xin[l], outs[l])
            graphs.append(g)
        torch.cuda.synchronize()

        def step(i):  # noqa: F811
            graphs[i % len(graphs)].replay()

    if args.parity and rank == 0 and world == 1:
        parity_check(layers[0], X[0])

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = Clocks(local) if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(args.steps):
        step(args.warmup + i)
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = clk.stop() if clk else None
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tok_bytes = shape.token_bytes()
    gbs = args.steps * tok_bytes / (ms / 1e3) / 1e9
    launches_per_step = 4   # router, gate/up, down, then combine (N = 1) or the NVLink slot exchange (N > 1)

    # ---- per-kernel live timing (same workload, events between launches) ----
    kt = per_kernel_times(layers, X, args, world, group)
    peak, peak_kind = peak_hbm()
    s = shape
    from sepia_b200 import quants as Q
    gu_bytes = (s.topk * s.ff * (Q.row_bytes(s.gate_type, s.hidden) + Q.row_bytes(s.up_type, s.hidden))
                + s.n_shared * s.ff * (Q.row_bytes(s.sh_gate_type, s.hidden) + Q.row_bytes(s.sh_up_type, s.hidden))
                + 4 * s.hidden + 4 * (s.topk + s.n_shared) * s.ff)
    dn_bytes = (s.topk * s.hidden * Q.row_bytes(s.down_type, s.ff) + s.n_shared * s.hidden * Q.row_bytes(s.sh_down_type, s.ff)
                + 4 * (s.topk + s.n_shared) * s.ff + 4 * s.hidden)
    rt_bytes = s.router_bytes() + 4 * s.n_routed + 4 * s.hidden
    roof = None
    if kt and world == 1:
        ach = gu_bytes / (kt["k_gateup"] / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": "k_gateup", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                "frac": round(ach / peak, 4), "peak_kind": peak_kind, "traffic": committed_traffic(),
                "algorithmic_bytes_per_launch": gu_bytes,
                "per_kernel_us": {k: round(v * 1e3, 2) for k, v in kt.items()},
                "per_kernel_gbs": {"k_router": round(rt_bytes / (kt["k_router"] / 1e3) / 1e9, 1),
                                   "k_gateup": round(ach, 1),
                                   "k_down": round(dn_bytes / (kt["k_down"] / 1e3) / 1e9, 1)}}

    # ---- e2e through the C ABI with host buffers ----
    e2e = None
    if not args.no_e2e and world == 1:
        e2e = abi_e2e(layers, args, shape)
    elif world > 1:
        e2e = sharded_e2e(layers, args, shape, group)

    # ---- config 5: whole-model decode (the layers above are freed first) ----
    decode = None
    if not args.no_decode:
        del layers, graphs
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        decode = decode_measure(args, world, rank, group)

    # ---- the other BASELINE kernels (configs 1, 3, 4) and the real-format layer ----
    kernels = None
    if world == 1 and not args.no_kernels:
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        kernels = {r["kernel"]: {k: r[k] for k in ("value", "us", "frac_of_measured_peak") if k in r}
                   for r in kernel_lines(args)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sec, n, sample, sec1 = cpu_token_seconds(shape)
        cpu = {"value": round(tok_bytes / sec / 1e9, 4), "unit": "GB/s", "cores": n, "kind": "port",
               "cpu_model": cpu_model(), "sample": sample, "layer_steps_per_s": round(1.0 / sec, 3),
               "one_thread": {"value": round(tok_bytes / sec1 / 1e9, 4), "unit": "GB/s", "cores": 1,
                              "layer_steps_per_s": round(1.0 / sec1, 4)}}

    if rank == 0:
        line = {"metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (BASELINE config 2 distributions, device-generated, seeded)",
                "config": {"workload": "config2_moe_layer_decode_1tok", "hidden": 7168, "ff": 2048, "experts": 256,
                           "topk": 6, "shared": 2, "types": "Q2_K gate/up, Q3_K down, Q4_K shared, f32 router",
                           "parallelism": f"ep{world}" if world > 1 else "single", "layer_instances": args.layers,
                           "l2": f"inputs larger than L2: {args.layers} rotating layer instances x "
                                 f"{tok_bytes / 1e6:.1f} MB/step", "bytes_per_token": tok_bytes},
                "pct_of_8tbs": round(100 * gbs / 8000, 2), "pct_of_measured_peak": round(100 * gbs / peak, 2),
                "layer_steps_per_s": round(args.steps / (ms / 1e3), 1),
                "roofline": roof, "e2e": e2e, "cpu_baseline": cpu, "gpu_launches": launches_per_step * args.steps,
                "clocks": clocks, "decode": decode, "kernels": kernels}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def per_kernel_times(layers, X, args, world, group):
    """Average device time of each kernel of the layer, CUDA events on the
    launching stream, over `steps` steps of the same rotation."""
    import torch
    from sepia_b200.lib import load, ok
    L = load()
    st = torch.cuda.current_stream()
    n = max(20, min(args.steps, 200))
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n)]
    out = torch.empty(layers[0].shape.hidden, device="cuda")
    # hold the device back while the host enqueues every launch, so that the
    # events bracket device time only (no host launch gaps)
    torch.cuda._sleep(100_000_000)
    for i in range(n):
        D = layers[i % len(layers)]
        x = X[i % 64]
        Ls, ws = C.byref(D.struct), C.byref(D.ws)
        ev[i][0].record(st)
        ok(L.sepia_cuda_moe_router(Ls, x.data_ptr(), ws, st.cuda_stream))
        ev[i][1].record(st)
        ok(L.sepia_cuda_moe_gateup(Ls, x.data_ptr(), ws, st.cuda_stream))
        ev[i][2].record(st)
        ok(L.sepia_cuda_moe_down(Ls, ws, out.data_ptr(), 1 if world > 1 else 0, st.cuda_stream))
        ev[i][3].record(st)
    torch.cuda.synchronize()
    names = ["k_router", "k_gateup", "k_down"]
    tot = {k: 0.0 for k in names}
    for i in range(n):
        for j, k in enumerate(names):
            tot[k] += ev[i][j].elapsed_time(ev[i][j + 1])
    return {k: v / n for k, v in tot.items()}


def abi_e2e(layers, args, shape):
    """Per step: write x into a Shared buffer's host mirror, sepia_gpu_begin
    (uploads it), sepia_gpu_moe_layer, sepia_gpu_end (downloads the output,
    waits), read the output on the host. Weights sit in Private buffers."""
    import numpy as np
    import torch
    from cuda.bindings import runtime as rt
    from sepia_b200.lib import SepiaGpuMoeDesc, load
    from sepia_b200.synth import hidden_state
    G = load()
    assert G.sepia_gpu_init(b"cuda") == 1
    s = shape
    sg, su, sd, ssg, ssu, ssd = s.strides()
    descs, bufs = [], []

    def dev_copy(dst_buf, dst_off, src_t):
        ptr = G.sepia_gpu_gpu_addr(dst_buf) + dst_off
        err, = rt.cudaMemcpy(ptr, src_t.data_ptr(), src_t.numel() * src_t.element_size(),
                             rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
        assert err == rt.cudaError_t.cudaSuccess

    for D in layers:
        ne = D.gate.numel() + D.up.numel() + D.down.numel()
        nsh = D.sh_gate.numel() + D.sh_up.numel() + D.sh_down.numel()
        be, bsh = G.sepia_gpu_alloc(ne, 1), G.sepia_gpu_alloc(nsh, 1)
        brw, brb = G.sepia_gpu_alloc(D.router_w.numel() * 4, 1), G.sepia_gpu_alloc(D.router_bias.numel() * 4, 1)
        assert be and bsh and brw and brb
        dev_copy(be, 0, D.gate)
        dev_copy(be, D.gate.numel(), D.up)
        dev_copy(be, D.gate.numel() + D.up.numel(), D.down)
        dev_copy(bsh, 0, D.sh_gate)
        dev_copy(bsh, D.sh_gate.numel(), D.sh_up)
        dev_copy(bsh, D.sh_gate.numel() + D.sh_up.numel(), D.sh_down)
        dev_copy(brw, 0, D.router_w)
        dev_copy(brb, 0, D.router_bias)
        d = SepiaGpuMoeDesc()
        d.hidden, d.ff, d.n_routed, d.n_shared, d.topk = s.hidden, s.ff, s.n_routed, s.n_shared, s.topk
        d.route_scale, d.global_scale = s.route_scale, s.global_scale
        d.router_w, d.router_bias = brw, brb
        d.gate_type, d.up_type, d.down_type = s.gate_type, s.up_type, s.down_type
        d.experts, d.gate_off, d.up_off, d.down_off = be, 0, D.gate.numel(), D.gate.numel() + D.up.numel()
        d.gate_stride, d.up_stride, d.down_stride = sg, su, sd
        d.sh_gate_type, d.sh_up_type, d.sh_down_type = s.sh_gate_type, s.sh_up_type, s.sh_down_type
        d.shared, d.sh_gate_off, d.sh_up_off = bsh, 0, D.sh_gate.numel()
        d.sh_down_off = D.sh_gate.numel() + D.sh_up.numel()
        d.sh_gate_stride, d.sh_up_stride, d.sh_down_stride = ssg, ssu, ssd
        descs.append(d)
        bufs += [be, bsh, brw, brb]
    xs = [hidden_state(i, s.hidden) for i in range(1, 65)]
    bx, bo = G.sepia_gpu_alloc(s.hidden * 4, 0), G.sepia_gpu_alloc(s.hidden * 4, 0)
    hx, ho = G.sepia_gpu_host_ptr(bx), G.sepia_gpu_host_ptr(bo)
    res = np.empty(s.hidden, np.float32)
    chk = 0.0

    def step(i):
        nonlocal chk
        C.memmove(hx, xs[i % 64].ctypes.data, s.hidden * 4)
        assert G.sepia_gpu_begin() == 1
        assert G.sepia_gpu_moe_layer(C.byref(descs[i % len(descs)]), bx, bo, None, None) == 1
        assert G.sepia_gpu_end() == 1
        C.memmove(res.ctypes.data, ho, s.hidden * 4)
        chk += float(res[0])

    torch.cuda.synchronize()
    for i in range(max(3, args.warmup)):
        step(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = time.perf_counter() - t0
    for b in bufs + [bx, bo]:
        G.sepia_gpu_free(b)
    return {"value": round(args.steps * s.token_bytes() / dt / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": s.hidden * 4, "d2h_bytes_per_step": s.hidden * 4,
            "ms_per_step": round(1e3 * dt / args.steps, 4), "tok_s": round(args.steps / dt, 1),
            "path": "sepia_gpu_begin + sepia_gpu_moe_layer + sepia_gpu_end (host-buffer ABI)"}


def sharded_e2e(layers, args, shape, group):
    """N > 1: pinned host x -> device, the sharded layer (router, own experts,
    NVLink slot exchange + combine), device -> pinned host output; wall clock
    per step, max over ranks."""
    import torch
    import torch.distributed as dist
    from sepia_b200.synth import hidden_state
    s = shape
    hx = [torch.from_numpy(hidden_state(i, s.hidden)).pin_memory() for i in range(1, 65)]
    ho = torch.empty(s.hidden, dtype=torch.float32).pin_memory()
    xd = torch.empty(s.hidden, dtype=torch.float32, device="cuda")
    out = torch.empty(s.hidden, dtype=torch.float32, device="cuda")

    def step(i):
        xd.copy_(hx[i % 64], non_blocking=True)
        layers[i % len(layers)].forward(xd, out, group=group)
        ho.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(max(3, args.warmup)):
        step(i)
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(i)
    dt = torch.tensor([time.perf_counter() - t0], device="cuda")
    dist.all_reduce(dt, op=dist.ReduceOp.MAX)
    dt = float(dt.item())
    return {"value": round(args.steps * s.token_bytes() / dt / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": s.hidden * 4, "d2h_bytes_per_step": s.hidden * 4,
            "ms_per_step": round(1e3 * dt / args.steps, 4), "tok_s": round(args.steps / dt, 1),
            "path": "sepia_cuda_moe_layer_sharded (router, owned experts, one-kernel NVLink slot exchange)"}


def parity_check(D, x):
    """One step of the bench's own device-generated layer against the oracle
    (the selected experts are copied back to the host)."""
    import numpy as np
    import torch
    from oracle import oracle as O
    out = torch.empty(D.shape.hidden, device="cuda")
    D.forward(x, out)
    torch.cuda.synchronize()
    idx = D.topk_idx.cpu().numpy()
    s = D.shape
    xh = x.cpu().numpy()
    logits = O.linear(D.router_w.cpu().numpy(), xh)
    ri, rw = O.route_select(logits, D.router_bias.cpu().numpy(), s.n_routed, s.n_shared, s.topk, s.route_scale,
                            s.global_scale)
    assert np.array_equal(ri, idx), (ri, idx)
    ref = np.zeros(s.hidden, np.float32)
    for j, e in enumerate(idx):
        g, u, d = D.expert_bytes_host(int(e))
        ref += O.expert_swiglu(s.gate_type, g, s.up_type, u, s.down_type, d, s.hidden, s.ff, xh, nthreads=8) * rw[j]
    sg, su, sd = D.strides[3:]
    for k in range(s.n_shared):
        from sepia_b200 import quants as Q
        ng = Q.row_bytes(s.sh_gate_type, s.hidden) * s.ff
        nu = Q.row_bytes(s.sh_up_type, s.hidden) * s.ff
        nd = Q.row_bytes(s.sh_down_type, s.ff) * s.hidden
        ref += O.expert_swiglu(s.sh_gate_type, D.sh_gate[k * sg:k * sg + ng].cpu().numpy(), s.sh_up_type,
                               D.sh_up[k * su:k * su + nu].cpu().numpy(), s.sh_down_type,
                               D.sh_down[k * sd:k * sd + nd].cpu().numpy(), s.hidden, s.ff, xh, rw[s.topk + k],
                               nthreads=8)
    err = O.rel_err(out.cpu().numpy(), ref)
    print(f"parity: router ids {list(idx)} match; max_rel_err {err:.2e}", file=sys.stderr)
    assert err <= 1e-4


if __name__ == "__main__":
    main()
