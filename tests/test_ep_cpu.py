"""Expert-parallel exchange logic (zmoe.ep) on CPU ranks over gloo: counts
all-to-all, row all-to-all, regroup by local expert, results back, combine.
Every rank's output must match the single-process oracle layer on its tokens."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from zmoe import ep
from zmoe import synthetic as syn

QWEN_S = syn.LayerShape(hidden=256, num_experts=8, inter=64, topk=4, kind=0, shared_inter=128, shared_gate=True)
DS_S = syn.LayerShape(hidden=256, num_experts=12, inter=96, topk=3, kind=0, shared_inter=192, shared_gate=False)
SW_S = syn.LayerShape(hidden=256, num_experts=8, inter=128, topk=1, kind=1, capacity=3, seq_len=16)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_and_regroup_plan():
    p = ep.ExpertPartition(60, 8)
    assert p.sizes() == [7, 8, 7, 8, 7, 8, 7, 8] and p.bounds[-1] == 60
    assert [p.owner(e) for e in (0, 6, 7, 59)] == [0, 0, 1, 7]
    rc = np.array([[2, 0, 1], [1, 3, 0]])        # [src][local expert]
    index, inverse, cl = ep.regroup_plan(rc)
    # received order: s0e0 s0e0 s0e2 s1e0 s1e1 s1e1 s1e1 -> grouped: e0(s0,s0,s1) e1(s1 x3) e2(s0)
    assert index.tolist() == [0, 1, 3, 4, 5, 6, 2]
    assert cl.tolist() == [3, 3, 1]
    assert (index[inverse] == np.arange(7)).all()
    empty = ep.regroup_plan(np.zeros((2, 3), int))
    assert empty[0].size == 0 and empty[2].tolist() == [0, 0, 0]


def _worker(rank, world, port, shape_name, tokens, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ep_oracle_kernels import OracleKernels, OracleLocalExperts
        from oracle import moe
        s = {"qwen": QWEN_S, "deepseek": DS_S, "switch": SW_S}[shape_name]
        w = syn.expert_weights(s, 1, std=0.05, seed=10)[0]
        wr, sg = syn.router_weights(s, std=0.05, seed=12)
        sh = syn.shared_weights(s, std=0.05, seed=14)
        bias = torch.linspace(0.0, -1.5, s.num_experts)
        x = syn.activations(tokens, s.hidden, seed=20 + rank)
        part = ep.ExpertPartition(s.num_experts, world)
        local = OracleLocalExperts(s, [w[e] for e in part.owned(rank)])
        layer = ep.EPMoELayer(s, OracleKernels(s, wr, bias, sg, sh), local)
        out = layer(x)
        if s.kind == 1:
            ref, _ = moe.switch_layer(x, wr, w, s.capacity, s.seq_len, bias=bias.numpy())
        elif s.shared_gate:
            ref, _ = moe.qwen_layer(x, wr, w, sh, sg, s.topk, bias=bias.numpy())
        else:
            ref, _ = moe.deepseek_layer(x, wr, w, sh, s.topk, s.scaling, bias=bias.numpy())
        assert out.shape == ref.shape == (tokens, s.hidden)
        if tokens == 0:
            q.put((rank, 0.0, 0.0))
            return
        d = (out.float() - ref.float()).abs()
        q.put((rank, float(d.max()), float(d.mean() / ref.float().abs().mean())))
    except Exception as e:                      # report, never hang the parent
        q.put((rank, repr(e), None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("shape_name,world,tokens", [("qwen", 2, 24), ("deepseek", 3, 20), ("switch", 2, 32),
                                                     ("qwen", 3, 0), ("deepseek", 4, 5)])
def test_ep_matches_single_process_layer(shape_name, world, tokens):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shape_name, tokens, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, mx, rel in res:
        assert rel is not None, f"rank {rank}: {mx}"
        assert mx <= 2e-2 and (tokens == 0 or rel <= 5e-3), (rank, mx, rel)
