"""GPU parity at the benchmark shapes, against the oracle.

* Qwen1.5-MoE-A2.7B layer: hidden 2048, 60 experts (SwiGLU, intermediate
  1408), top-4 softmax, shared expert 5632 with a sigmoid gate, Zipf(1.0)
  router bias, LZ4HC-9 in 3 chunks per matrix, 16 cached experts; one layer
  forwarded at 1, 16, 128 and 512 tokens in turn (hits, misses and evictions
  all happen).
* DeepSeek-V2-Lite layer: 64 experts, top-6, routed_scaling 1.0, shared
  experts of combined intermediate 2816 (no gate), Zipf(1.2); 1 and 64 tokens.
* Switch-large-128 layer: d_model 1024, 128 ReLU experts of 2816, top-1 with
  capacity floor(1.25 * 4096 / 128) = 40 over one 4096-token sequence,
  overflow tokens passed through.
* The grouped FFN alone at the Qwen and Switch expert shapes, with groups of
  0, 1, 129, 256, 300 and 512 rows (several token tiles) and more groups than
  one launch takes (70 SwiGLU groups, 130 ReLU groups: split launches).

Router logits, top-k indices and weights, per-expert counts and permuted rows
are compared bit for bit; layer outputs within max-abs 2e-2 and mean-rel 5e-3
of the oracle's fp32-accumulate path."""
import numpy as np
import pytest
import torch

from oracle import moe
from zmoe import synthetic as syn

pytestmark = pytest.mark.gpu
TOL_MAX_ABS = 2e-2
TOL_MEAN_REL = 5e-3


def _close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.abs(a - b)
    return d.max(), d.mean() / max(np.abs(b).mean(), 1e-12)


def _layer(s, max_tokens, cache, codec="LZ4HC", level=9, bias=None):
    from zmoe.layer import MoELayer
    w = syn.expert_weights(s, 1)[0]
    wr, sg = syn.router_weights(s)
    sh = syn.shared_weights(s)
    L = MoELayer(s, max_tokens=max_tokens, cache_slots=cache)
    L.set_router(wr, bias, sg)
    if sh is not None:
        L.set_shared(*sh)
    L.load_experts(w, num_file_chunks=3, codec=codec, level=level)
    return L, w, wr, sg, sh


def _check_routing(s, x, wr, sg, bias, r, mode):
    """Router outputs and permuted counts of the product against the oracle route r."""
    from zmoe import ops
    xd = x.cuda()
    logits, idx, tw, g = ops.router(xd, wr.cuda(), s.topk, mode, bias.cuda() if bias is not None else None,
                                    sg.cuda() if sg is not None else None, scaling=s.scaling)
    cap = s.capacity if mode == ops.ROUTE_SWITCH else 0
    counts, offsets, row_of, tor, xp = ops.permute(idx, xd, s.num_experts, cap, s.seq_len if cap else 0)
    torch.cuda.synchronize()
    assert np.array_equal(logits.cpu().numpy(), r.logits)
    assert np.array_equal(idx.cpu().numpy(), r.topk_idx)
    assert np.array_equal(tw.cpu().numpy(), r.topk_w)
    assert np.array_equal(counts.cpu().numpy(), r.counts)
    offs, tor_ref, row_ref = moe.permute(r.topk_idx, s.num_experts)
    assert np.array_equal(row_of.cpu().numpy(), row_ref)
    n = int(offs[-1])
    assert torch.equal(xp[:n].cpu(), x[torch.from_numpy(tor_ref).long()])


@pytest.fixture(scope="module")
def qwen_layer():
    s = syn.QWEN
    bias = syn.zipf_bias(s, 0)
    L, w, wr, sg, sh = _layer(s, 512, 16, bias=bias)
    L.warm_cache(syn.popularity_order(s, 0)[:16])
    yield s, L, w, wr, sg, sh, bias
    L.close()


@pytest.mark.parametrize("T", [1, 16, 128, 512])
def test_qwen_layer_full_shape(qwen_layer, T):
    from zmoe import ops
    s, L, w, wr, sg, sh, bias = qwen_layer
    x = syn.activations(T, s.hidden, seed=100 + T)
    before = L.stats()
    out = L(x.cuda())
    L.sync()
    ref, r = moe.qwen_layer(x, wr, w, sh, sg, k=s.topk, bias=bias.numpy())
    mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
    assert mx <= TOL_MAX_ABS and mr <= TOL_MEAN_REL, (T, mx, mr)
    _check_routing(s, x, wr, sg, bias, r, ops.ROUTE_QWEN)
    st = L.stats()
    assert st["decode_errors"] == 0
    assert st["hits"] + st["misses"] - before["hits"] - before["misses"] == int((r.counts > 0).sum())
    if T == 512:
        assert st["misses"] > before["misses"]       # experts outside the cache were decoded in the step


@pytest.mark.parametrize("T", [1, 64])
def test_deepseek_layer_full_shape(T):
    from zmoe import ops
    s = syn.DEEPSEEK
    bias = syn.zipf_bias(s, 0)
    L, w, wr, _, sh = _layer(s, 64, 16, codec="LZ4", level=5, bias=bias)
    try:
        for t in (T, T):                              # the second call hits what the first decoded
            x = syn.activations(t, s.hidden, seed=200 + t)
            out = L(x.cuda())
            L.sync()
            ref, r = moe.deepseek_layer(x, wr, w, sh, k=s.topk, routed_scaling_factor=s.scaling,
                                        bias=bias.numpy())
            mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
            assert mx <= TOL_MAX_ABS and mr <= TOL_MEAN_REL, (t, mx, mr)
            _check_routing(s, x, wr, None, bias, r, ops.ROUTE_DEEPSEEK)
        assert L.stats()["decode_errors"] == 0
    finally:
        L.close()


def test_switch_layer_full_shape_capacity():
    from zmoe import ops
    s = syn.SWITCH
    assert s.capacity == (125 * 4096) // (100 * 128) and s.seq_len == 4096
    L, w, wr, _, _ = _layer(s, 4096, 16, codec="LZ4", level=5)
    try:
        x = syn.activations(4096, s.hidden, seed=300)
        out = L(x.cuda())
        L.sync()
        ref, r = moe.switch_layer(x, wr, w, s.capacity, s.seq_len)
        assert (r.topk_idx < 0).any() and r.counts.max() <= s.capacity
        mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
        assert mx <= TOL_MAX_ABS and mr <= TOL_MEAN_REL, (mx, mr)
        r.topk_idx = r.topk_idx.copy()
        _check_switch_routing(s, x, wr, r)
    finally:
        L.close()


def _check_switch_routing(s, x, wr, r):
    from zmoe import ops
    xd = x.cuda()
    logits, idx, tw, _ = ops.router(xd, wr.cuda(), 1, ops.ROUTE_SWITCH)
    counts, offsets, row_of, tor, xp = ops.permute(idx, xd, s.num_experts, s.capacity, s.seq_len)
    torch.cuda.synchronize()
    assert np.array_equal(logits.cpu().numpy(), r.logits)
    assert np.array_equal(idx.cpu().numpy(), r.topk_idx)       # -1 where the capacity dropped the token
    assert np.array_equal(tw.cpu().numpy(), r.topk_w)
    assert np.array_equal(counts.cpu().numpy(), r.counts)


def _groups(n_groups, special):
    rows = [(g * 37) % 7 for g in range(n_groups)]
    for g, v in special.items():
        rows[g] = v
    return rows


@pytest.mark.parametrize("kind,G,H,I", [(0, 64, 2048, 1408), (0, 70, 2048, 1408), (1, 128, 1024, 2816),
                                        (1, 130, 1024, 2816)])
def test_grouped_ffn_large_groups_and_split_launches(kind, G, H, I):
    from zmoe import ops
    rows = _groups(G, {0: 0, 1: 1, 5: 129, 17: 256, G - 7: 300, G - 1: 512})
    gen = torch.Generator().manual_seed(40 + G + kind)
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    R = int(offs[-1])
    x = torch.randn(R, H, generator=gen).to(torch.bfloat16)
    pool = []                                  # 6 distinct weight sets, shared round robin by the groups
    for _ in range(6):
        if kind == 0:
            pool.append([(torch.randn(I, H, generator=gen) * 0.02).to(torch.bfloat16),
                         (torch.randn(I, H, generator=gen) * 0.02).to(torch.bfloat16),
                         (torch.randn(H, I, generator=gen) * 0.02).to(torch.bfloat16)])
        else:
            pool.append([(torch.randn(I, H, generator=gen) * 0.02).to(torch.bfloat16), None,
                         (torch.randn(H, I, generator=gen) * 0.02).to(torch.bfloat16)])
    dev = [[t.cuda() if t is not None else None for t in m] for m in pool]
    wtab = ops.weight_table([dev[g % 6] for g in range(G)], "cuda")
    y, _ = ops.expert_ffn(x.cuda(), wtab, torch.from_numpy(offs).cuda(), G, I, kind)
    torch.cuda.synchronize()
    got = y.float().cpu()
    for g in range(G):
        a, b = int(offs[g]), int(offs[g + 1])
        if a == b:
            continue
        m = pool[g % 6]
        ref = moe.swiglu_fp32(x[a:b], *m) if kind == 0 else moe.relu_ffn_fp32(x[a:b], m[0], m[2])
        mx, mr = _close(got[a:b].numpy(), ref.numpy())
        assert mx <= TOL_MAX_ABS and mr <= TOL_MEAN_REL, (g, b - a, mx, mr)


def test_shared_expert_shape_one_group_512_rows():
    """The Qwen shared expert: one group (no offsets) of 512 rows, I = 5632."""
    from zmoe import ops
    s = syn.QWEN
    sh = syn.shared_weights(s)
    x = syn.activations(512, s.hidden, seed=400)
    dev = [t.cuda() for t in sh]
    y, _ = ops.expert_ffn(x.cuda(), ops.weight_table([dev], "cuda"), None, 1, s.shared_inter, 0)
    torch.cuda.synchronize()
    ref = moe.swiglu_fp32(x, *sh)
    mx, mr = _close(y.float().cpu().numpy(), ref.numpy())
    assert mx <= TOL_MAX_ABS and mr <= TOL_MEAN_REL, (mx, mr)
