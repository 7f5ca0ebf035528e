"""CPU, world size 2 over gloo: the expert-sharding protocol of the MoE layer.

Every rank runs the same router, computes only the experts it owns
(sepia_b200.moe.owned_experts / owned_shared: routed expert e on rank
e % world, shared expert s on rank s % world), writes each owned slot's term
into a [topk + n_shared, hidden] buffer that is zero elsewhere, sums the
buffers with an all-reduce and combines the slots in the reference's order
(routed j = 0..k-1, then shared; mlp_moe_forward, src/sepia.c:1377-1470).
The result must equal the single-process layer bit for bit: only one rank
contributes each slot, so the all-reduce adds exact zeros. The expert math is
the oracle's CPU restatement; the GPU run of the same protocol is in
test_gpu_moe.py.
"""
import os
import socket

import numpy as np
import torch.multiprocessing as mp

from sepia_b200.synth import MoeShape, hidden_state, moe_layer_host

SHAPE = MoeShape(hidden=512, ff=256, n_routed=16, n_shared=2, topk=4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_terms(H, x, rank, world):
    from oracle import oracle as O
    from sepia_b200.moe import owned_experts, owned_shared
    _, _, idx, w = O.moe_layer(H, x)
    n_slots = H.topk + H.n_shared
    slots = np.zeros((n_slots, H.hidden), np.float32)
    mine = set(owned_experts(H.n_routed, rank, world))
    for j, e in enumerate(idx):
        if int(e) in mine:
            g = H.gate[int(e) * H.gate_stride:]
            u = H.up[int(e) * H.up_stride:]
            d = H.down[int(e) * H.down_stride:]
            eo = O.expert_swiglu(H.gate_type, g, H.up_type, u, H.down_type, d, H.hidden, H.ff, x)
            slots[j] = eo * np.float32(w[j])
    for s in owned_shared(H.n_shared, rank, world):
        g = H.sh_gate[s * H.sh_gate_stride:]
        u = H.sh_up[s * H.sh_up_stride:]
        d = H.sh_down[s * H.sh_down_stride:]
        slots[H.topk + s] = O.expert_swiglu(H.sh_gate_type, g, H.sh_up_type, u, H.sh_down_type, d, H.hidden, H.ff,
                                            x, float(w[H.topk + s]))
    return slots


def _combine(slots):
    out = np.zeros(slots.shape[1], np.float32)
    for s in range(slots.shape[0]):
        out = (out + slots[s]).astype(np.float32)
    return out


def _worker(rank, world, port, seeds, q):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    H = moe_layer_host(SHAPE, seed=5)
    outs = []
    for seed in seeds:
        x = hidden_state(seed, SHAPE.hidden)
        t = torch.from_numpy(_rank_terms(H, x, rank, world))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        outs.append(_combine(t.numpy()))
    dist.destroy_process_group()
    q.put((rank, outs))


def test_sharded_layer_matches_single_process():
    from oracle import oracle as O
    O.build()
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    seeds = [1, 2, 7]
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seeds, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    H = moe_layer_host(SHAPE, seed=5)
    for i, seed in enumerate(seeds):
        want = O.moe_layer(H, hidden_state(seed, SHAPE.hidden))[0]
        for r in range(world):
            np.testing.assert_array_equal(got[r][i], want)


def test_every_expert_has_one_owner():
    from sepia_b200.moe import owned_experts, owned_shared
    for world in (1, 2, 4, 8):
        routed = sorted(e for r in range(world) for e in owned_experts(256, r, world))
        assert routed == list(range(256))
        shared = sorted(s for r in range(world) for s in owned_shared(2, r, world))
        assert shared == [0, 1]
