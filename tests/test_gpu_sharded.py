"""GPU, several devices: expert sharding with the one-kernel NVLink slot
exchange (sepia_cuda_exchange_*, sepia_model_connect). One process per GPU;
the handles travel over a gloo process group. Skipped when the box has fewer
GPUs than ranks: ranks that wait on each other never share a GPU.

  - one MoE layer, sharded over world ranks, equals the one-GPU layer bit
    for bit (router ids, output) over several tokens, eager and replayed
    from a CUDA graph;
  - the whole model (tests/golden/model_*.npz containers) decodes the
    reference's greedy ids token-exactly on every rank."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _layer_worker(rank, world, port, q):
    try:
        import torch
        sys.path.insert(0, str(HERE.parent))
        _init(rank, world, port)
        from sepia_b200.moe import Exchange, MoeLayerDevice
        from sepia_b200.synth import MoeShape, hidden_state
        shape = MoeShape(hidden=2048, ff=512, n_routed=32)
        full = MoeLayerDevice.random(shape, seed=9)
        mine = MoeLayerDevice.random(shape, seed=9, rank=rank, world=world)
        mine.exchange = Exchange(shape.topk + shape.n_shared, shape.hidden, rank, world)
        mine.exchange.connect()
        res = []
        x = torch.empty(shape.hidden, device="cuda")
        a = torch.empty(shape.hidden, device="cuda")
        b = torch.empty(shape.hidden, device="cuda")
        for seed in (1, 2, 3, 40):
            x.copy_(torch.from_numpy(hidden_state(seed, shape.hidden)))
            full.forward(x, a)
            mine.forward(x, b)
            torch.cuda.synchronize()
            res.append(bool(torch.equal(a.view(torch.int32), b.view(torch.int32))) and
                       bool(torch.equal(full.topk_idx, mine.topk_idx)))
        # the same step replayed from a CUDA graph, several times in a row
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            mine.forward(x, b)
        for seed in (5, 6, 7):
            x.copy_(torch.from_numpy(hidden_state(seed, shape.hidden)))
            full.forward(x, a)
            g.replay()
            torch.cuda.synchronize()
            res.append(bool(torch.equal(a.view(torch.int32), b.view(torch.int32))))
        from sepia_b200.lib import load
        res.append(load().sepia_cuda_device_error(None) == 0)
        q.put((rank, res))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


def _model_worker(rank, world, port, cdir, prompt, n_gen, q):
    try:
        sys.path.insert(0, str(HERE.parent))
        _init(rank, world, port)
        from sepia_b200.model import DeviceModel
        m = DeviceModel.from_container(cdir, max_positions=128, rank=rank, world=world)
        m.connect()
        ids = m.generate(prompt, n_gen)
        ids2 = m.generate(prompt, n_gen)
        q.put((rank, [ids.tolist(), ids2.tolist()]))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def _run(world, target, *args):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=600)
            out[r] = v
    finally:
        for p in ps:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return out


def _need(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_layer_bit_identical(lib, world):
    _need(world)
    out = _run(world, _layer_worker)
    for r in range(world):
        assert isinstance(out[r], list) and all(out[r]), (r, out[r])


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_model_token_exact(lib, tmp_path, world):
    _need(world)
    sys.path.insert(0, str(HERE / "golden"))
    import make_model_golden as G
    fx = np.load(HERE / "golden" / "model_baseline_types.npz")
    d, prompt, digest = G.build("baseline_types", tmp_path / "m")
    assert digest == str(fx["digest"])
    out = _run(world, _model_worker, str(d), prompt, len(fx["ids"]))
    for r in range(world):
        assert isinstance(out[r], list), (r, out[r])
        assert out[r][0] == fx["ids"].tolist() and out[r][1] == fx["ids"].tolist(), (r, out[r])
