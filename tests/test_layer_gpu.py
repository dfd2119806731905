"""GPU parity of router / permute / expert FFN / combine and of whole layers
against the oracle (bit-exact for indices, counts, rows and router logits;
max-abs 2e-2 and mean-rel 5e-3 for layer outputs)."""
import numpy as np
import pytest
import torch

from oracle import moe
from zmoe import synthetic as syn

pytestmark = pytest.mark.gpu
TOL_MAX_ABS = 2e-2
TOL_MEAN_REL = 5e-3


def _ops():
    from zmoe import ops
    return ops


def _close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.abs(a - b)
    return d.max(), d.mean() / max(np.abs(b).mean(), 1e-12)


@pytest.mark.parametrize("mode,E,k,H,T", [(0, 60, 4, 2048, 67), (1, 64, 6, 2048, 33), (2, 128, 1, 1024, 40),
                                          (0, 8, 4, 256, 5), (1, 17, 3, 512, 1)])
def test_router_bit_exact(mode, E, k, H, T):
    ops = _ops()
    gen = torch.Generator().manual_seed(E * 7 + T)
    x = torch.randn(T, H, generator=gen).to(torch.bfloat16)
    w = (torch.randn(E, H, generator=gen) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(E, generator=gen) * 0.5).float()
    sg = (torch.randn(1, H, generator=gen) * 0.02).to(torch.bfloat16) if mode == 0 else None
    logits, idx, tw, g = ops.router(x.cuda(), w.cuda(), k, mode, bias.cuda(),
                                    sg.cuda() if sg is not None else None, scaling=1.0)
    torch.cuda.synchronize()
    if mode == 0:
        r = moe.route_qwen(x, w, k, bias=bias.numpy())
    elif mode == 1:
        r = moe.route_deepseek(x, w, k, 1.0, bias=bias.numpy())
    else:
        r = moe.route_switch(x, w, capacity=0, seq_len=T, bias=bias.numpy())
        r.topk_idx = r.extra["argmax"][:, None]
    assert np.array_equal(logits.cpu().numpy(), r.logits)
    assert np.array_equal(idx.cpu().numpy(), r.topk_idx)
    assert np.array_equal(tw.cpu().numpy(), r.topk_w)
    if sg is not None:
        ref = torch.sigmoid(torch.from_numpy(moe.bf16_round(moe.router_logits(moe.to_f32(x), moe.to_f32(sg))))).numpy()[:, 0]
        assert np.abs(g.cpu().numpy() - ref).max() < 1e-6


def test_router_tie_break_lower_index():
    ops = _ops()
    H, E, T = 256, 8, 4
    x = torch.ones(T, H, dtype=torch.bfloat16)
    w = torch.zeros(E, H, dtype=torch.bfloat16)
    w[3] = 0.01
    w[5] = 0.01                       # experts 3 and 5 tie; all others tie at 0
    _, idx, _, _ = ops.router(x.cuda(), w.cuda(), 4, 0)
    assert idx.cpu().tolist() == [[3, 5, 0, 1]] * T


@pytest.mark.parametrize("T,k,E,cap,seq", [(512, 4, 60, 0, 0), (37, 6, 64, 0, 0), (256, 1, 16, 10, 64), (1, 4, 60, 0, 0)])
def test_permute_exact(T, k, E, cap, seq):
    ops = _ops()
    rng = np.random.default_rng(T + E)
    idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    H = 256
    x = torch.randn(T, H).to(torch.bfloat16)
    ref_idx = idx.copy()
    if cap:
        for b in range(T // seq):
            seen = np.zeros(E, np.int64)
            for s in range(seq):
                t = b * seq + s
                e = ref_idx[t, 0]
                seen[e] += 1
                if seen[e] > cap:
                    ref_idx[t, 0] = -1
    offs, tor, row_of = moe.permute(ref_idx, E)
    d_idx = torch.from_numpy(idx).cuda()
    counts, offsets, r_of, t_of, xp = ops.permute(d_idx, x.cuda(), E, cap, seq)
    torch.cuda.synchronize()
    assert np.array_equal(d_idx.cpu().numpy(), ref_idx)
    assert np.array_equal(offsets.cpu().numpy(), offs)
    assert np.array_equal(counts.cpu().numpy(), np.diff(offs))
    assert np.array_equal(r_of.cpu().numpy(), row_of)
    n = int(offs[-1])
    assert np.array_equal(t_of.cpu().numpy()[:n], tor)
    assert torch.equal(xp[:n].cpu(), x[torch.from_numpy(tor).long()])


@pytest.mark.parametrize("kind", [0, 1])
def test_grouped_ffn_matches_oracle(kind):
    ops = _ops()
    gen = torch.Generator().manual_seed(11 + kind)
    H, I, G = 512, 192, 5
    rows = [0, 7, 1, 33, 16]
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    R = int(offs[-1])
    x = torch.randn(R, H, generator=gen).to(torch.bfloat16)
    mats = []
    for g in range(G):
        if kind == 0:
            mats.append([(torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16),
                         (torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16),
                         (torch.randn(H, I, generator=gen) * 0.05).to(torch.bfloat16)])
        else:
            mats.append([(torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16), None,
                         (torch.randn(H, I, generator=gen) * 0.05).to(torch.bfloat16)])
    dm = [[t.cuda() if t is not None else None for t in m] for m in mats]
    wtab = ops.weight_table(dm, "cuda")
    y, _ = ops.expert_ffn(x.cuda(), wtab, torch.from_numpy(offs).cuda(), G, I, kind)
    torch.cuda.synchronize()
    ref = torch.zeros(R, H)
    for g in range(G):
        a, b = offs[g], offs[g + 1]
        if b == a:
            continue
        if kind == 0:
            ref[a:b] = moe.swiglu_fp32(x[a:b], *mats[g])
        else:
            ref[a:b] = moe.relu_ffn_fp32(x[a:b], mats[g][0], mats[g][2])
    mx, mr = _close(y[:R].float().cpu().numpy(), ref.numpy())
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)


def run_layer_primitives(s: syn.LayerShape, x, wr, sg, experts, shared, bias=None):
    """Layer forward through the individual C-ABI primitives (decoded weights)."""
    ops = _ops()
    dev = "cuda"
    xd = x.cuda()
    mode = ops.ROUTE_SWITCH if s.kind == 1 else (ops.ROUTE_QWEN if s.shared_gate else ops.ROUTE_DEEPSEEK)
    _, idx, tw, g = ops.router(xd, wr.cuda(), s.topk, mode, bias.cuda() if bias is not None else None,
                               sg.cuda() if sg is not None else None, scaling=s.scaling)
    counts, offsets, row_of, tor, xp = ops.permute(idx, xd, s.num_experts, s.capacity if s.kind == 1 else 0,
                                                   s.seq_len if s.kind == 1 else 0)
    dm = [[t.cuda() for t in e] for e in experts]
    if s.kind == 1:
        dm = [[e[0], None, e[1]] for e in dm]
    wtab = ops.weight_table(dm, dev)
    y, _ = ops.expert_ffn(xp, wtab, offsets, s.num_experts, s.inter, s.kind, rows_total=xp.shape[0])
    ysh = None
    if shared is not None:
        st = ops.weight_table([[t.cuda() for t in shared]], dev)
        ysh, _ = ops.expert_ffn(xd, st, None, 1, s.shared_inter, 0)
    return ops.combine(y, row_of, tw, mode, ysh, g, xd)


def test_qwen_layer_small_matches_oracle_and_reference_run():
    import os
    from tests.golden.make_golden import QWEN_SMALL, small_inputs
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "qwen_block.npz"))
    s = QWEN_SMALL
    x, wr, sg, w, sh = small_inputs(s, int(gold["tokens"]))
    out = run_layer_primitives(s, x, wr, sg, w, sh)
    torch.cuda.synchronize()
    ref, _ = moe.qwen_layer(x, wr, w, sh, sg, k=s.topk)
    mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)
    mx, mr = _close(out.float().cpu().numpy(), gold["out"])
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)


def test_switch_layer_small_matches_oracle():
    s = syn.LayerShape(hidden=256, num_experts=8, inter=128, topk=1, kind=1, capacity=6, seq_len=32)
    w = syn.expert_weights(s, 1, std=0.05, seed=20)[0]
    wr, _ = syn.router_weights(s, std=0.05, seed=21)
    x = syn.activations(64, s.hidden, seed=22)
    out = run_layer_primitives(s, x, wr, None, w, None)
    torch.cuda.synchronize()
    ref, r = moe.switch_layer(x, wr, w, s.capacity, s.seq_len)
    assert (r.topk_idx < 0).any()
    mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)
