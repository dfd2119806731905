"""Expert parallelism on GPUs: the EP layer (zmoe.ep over the C ABI) must give
bit-identical outputs to the single-GPU layer engine on the same tokens (each
FFN row is independent of which rows share its group)."""
import os
import socket

import numpy as np
import pytest
import torch

from zmoe import synthetic as syn

pytestmark = pytest.mark.gpu

SHAPES = {
    "qwen": syn.LayerShape(hidden=256, num_experts=8, inter=64, topk=4, kind=0, shared_inter=128, shared_gate=True),
    "deepseek": syn.LayerShape(hidden=256, num_experts=12, inter=96, topk=3, kind=0, shared_inter=192),
    "switch": syn.LayerShape(hidden=256, num_experts=8, inter=128, topk=1, kind=1, capacity=3, seq_len=16),
}


def _inputs(s):
    from zmoe import codec as zc
    w = syn.expert_weights(s, 1, std=0.05, seed=10)[0]
    wr, sg = syn.router_weights(s, std=0.05, seed=12)
    sh = syn.shared_weights(s, std=0.05, seed=14)
    bias = torch.linspace(0.0, -1.5, s.num_experts)
    flat = zc.encode_tensors([t for e in w for t in e], 3)
    per = s.tensors_per_expert
    enc = [flat[e * per:(e + 1) * per] for e in range(s.num_experts)]
    return w, wr, sg, sh, bias, enc


def _single(s, wr, sg, sh, bias, enc, T, device=0):
    from zmoe.layer import MoELayer
    L = MoELayer(s, max_tokens=T, cache_slots=2, device=device)
    L.set_router(wr, bias, sg)
    if sh is not None:
        L.set_shared(*sh)
    for e, row in enumerate(enc):
        for t, et in enumerate(row):
            L.load_encoded(e, t, et)
    return L


@pytest.mark.parametrize("native", [True, False])
@pytest.mark.parametrize("name", ["qwen", "deepseek", "switch"])
def test_ep_one_rank_equals_layer_engine(name, native):
    from zmoe import ep
    s = SHAPES[name]
    w, wr, sg, sh, bias, enc = _inputs(s)
    T = 48
    x = syn.activations(T, s.hidden, seed=21).cuda()
    ref = _single(s, wr, sg, sh, bias, enc, T)(x)
    layer = ep.build_gpu_layer(s, enc, wr, bias, sg, sh, max_tokens=T, cache_slots=2, device=0, warm=[0, 1],
                               native=native)
    for _ in range(2):                                   # cold, then with cache state
        out = layer(x)
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def _rank(rank, world, port, name, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from zmoe import ep
        s = SHAPES[name]
        w, wr, sg, sh, bias, enc = _inputs(s)
        T = 32
        x = syn.activations(T, s.hidden, seed=30 + rank).cuda()
        ref = _single(s, wr, sg, sh, bias, enc, T, device=rank)(x)
        layer = ep.build_gpu_layer(s, enc, wr, bias, sg, sh, max_tokens=T, cache_slots=1, device=rank)
        ok = True
        for _ in range(2):
            out = layer(x)
            torch.cuda.synchronize()
            ok = ok and torch.equal(out.view(torch.int16), ref.view(torch.int16))
        q.put((rank, ok, None))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, False, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["qwen", "switch"])
def test_ep_two_ranks_nccl_equals_layer_engine(name):
    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, err in res:
        assert ok, (rank, err)
