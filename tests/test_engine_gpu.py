"""The C++ layer engine (compressed store in HBM, decoded cache, miss decode,
grouped FFN, combine) against the oracle layers."""
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


def _build(s, cache, transient=0, policy="ZipMoE", T=64, seed=0, bias=None):
    from zmoe.layer import MoELayer
    w = syn.expert_weights(s, 1, std=0.05, seed=seed)[0]
    wr, sg = syn.router_weights(s, std=0.05, seed=seed + 1)
    sh = syn.shared_weights(s, std=0.05, seed=seed + 2)
    L = MoELayer(s, max_tokens=T, cache_slots=cache, transient_slots=transient, policy=policy)
    L.set_router(wr, bias, sg)
    if sh is not None:
        L.set_shared(*sh)
    L.load_experts(w, num_file_chunks=3)
    return L, w, wr, sg, sh


QWEN_SMALL = syn.LayerShape(hidden=256, num_experts=8, inter=64, topk=4, kind=0, shared_inter=128, shared_gate=True)
DS_SMALL = syn.LayerShape(hidden=256, num_experts=12, inter=96, topk=3, kind=0, shared_inter=192, shared_gate=False)
SW_SMALL = syn.LayerShape(hidden=256, num_experts=8, inter=128, topk=1, kind=1, capacity=5, seq_len=32)


@pytest.mark.parametrize("cache,transient", [(2, 0), (0, 0), (8, 0), (2, 1), (3, 2)])
def test_engine_qwen_matches_oracle(cache, transient):
    s = QWEN_SMALL
    L, w, wr, sg, sh = _build(s, cache, transient)
    for step, T in enumerate([24, 1, 64, 24]):
        x = syn.activations(T, s.hidden, seed=100 + step)
        out = L(x.cuda())
        L.sync()
        ref, _ = moe.qwen_layer(x, wr, w, sh, sg, k=s.topk)
        mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
        assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (step, mx, mr)
    st = L.stats()
    assert st["forwards"] == 4 and st["decode_errors"] == 0
    assert st["hits"] + st["misses"] > 0
    if cache == 8:
        assert len(L.cached_experts()) == 8
    if cache == 0:
        assert st["hits"] == 0


def test_engine_deepseek_and_bias():
    s = DS_SMALL
    bias = torch.linspace(0, -2, s.num_experts)
    L, w, wr, _, sh = _build(s, 4, bias=bias)
    x = syn.activations(40, s.hidden, seed=7)
    out = L(x.cuda())
    L.sync()
    ref, _ = moe.deepseek_layer(x, wr, w, sh, k=s.topk, bias=bias.numpy())
    mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)


def test_engine_switch_capacity_passthrough():
    s = SW_SMALL
    L, w, wr, _, _ = _build(s, 2)
    x = syn.activations(64, s.hidden, seed=9)
    out = L(x.cuda())
    L.sync()
    ref, r = moe.switch_layer(x, wr, w, s.capacity, s.seq_len)
    assert (r.topk_idx < 0).any()
    mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)


def test_engine_cache_hits_follow_warm_set():
    s = QWEN_SMALL
    L, w, wr, sg, sh = _build(s, 8)
    L.warm_cache(range(8))
    x = syn.activations(32, s.hidden, seed=3)
    L(x.cuda())
    L.sync()
    st = L.stats()
    assert st["misses"] == 0 and st["hits"] > 0


def test_prefetch_does_not_wait_for_the_stream():
    # clock probes keep the current stream busy for 30 ms; prefetch must return
    # before they end, and the next forward must see the prefetched experts
    from zmoe._lib import lib
    s = QWEN_SMALL
    L, w, wr, sg, sh = _build(s, 4)
    x = syn.activations(32, s.hidden, seed=61)
    L(x.cuda())                                      # sizes the decoder scratch (a one-time synchronising allocation)
    L.sync()
    probe = torch.zeros(2, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(3):
        assert lib.zmoe_clock_probe(probe.data_ptr(), 10_000_000, stream.cuda_stream) == 0
    cached = set(L.cached_experts())
    want = [e for e in range(s.num_experts) if e not in cached][:2]
    L.prefetch(want)
    assert not stream.query()                        # the probe is still running: no host wait happened
    out = L(x.cuda())
    L.sync()
    assert set(want) <= set(L.cached_experts())
    ref, r = moe.qwen_layer(x, wr, w, sh, sg, k=s.topk)
    mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
    assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (mx, mr)
    st = L.stats()
    used = set(np.unique(r.topk_idx).tolist())
    assert st["hits"] >= len(used & set(want))


def test_overlapped_waves_match_oracle_over_many_forwards():
    # one transient slot: every miss beyond the cache is its own decode wave,
    # with the hit FFN running beside the first wave's decode
    s = QWEN_SMALL
    L, w, wr, sg, sh = _build(s, 3, transient=1, T=48)
    for step in range(6):
        x = syn.activations(8 + 8 * step, s.hidden, seed=70 + step)
        out = L(x.cuda())
        ref, _ = moe.qwen_layer(x, wr, w, sh, sg, k=s.topk)
        mx, mr = _close(out.float().cpu().numpy(), ref.float().numpy())
        assert mx < TOL_MAX_ABS and mr < TOL_MEAN_REL, (step, mx, mr)
    L.sync()
    assert L.stats()["decode_errors"] == 0


def test_engine_forward_host_matches_device():
    s = QWEN_SMALL
    L, *_ = _build(s, 2)
    x = syn.activations(16, s.hidden, seed=5)
    d = L(x.cuda()).cpu()
    xh = x.pin_memory()
    oh = torch.empty_like(xh).pin_memory()
    L.forward_host(xh, oh)
    assert torch.equal(d, oh)


def test_engine_host_store_matches_device_store():
    # compressed experts in pinned host memory, copied in per decode: the same
    # outputs as the HBM store, over several forwards with misses and evictions
    from zmoe.layer import MoELayer
    s = QWEN_SMALL
    L, w, wr, sg, sh = _build(s, 2)
    Lh = MoELayer(s, max_tokens=64, cache_slots=2, store="host")
    Lh.set_router(wr, None, sg)
    Lh.set_shared(*sh)
    Lh.load_experts(w, num_file_chunks=3)
    for i in range(4):
        x = syn.activations(16 + 8 * i, s.hidden, seed=40 + i).cuda()
        assert torch.equal(L(x), Lh(x))
    st, sth = L.stats(), Lh.stats()
    assert sth["misses"] == st["misses"] > 0
    assert sth["host_copy_bytes"] > 0 and st["host_copy_bytes"] == 0
    from zmoe._lib import ZmoeError, check, lib
    with pytest.raises(ZmoeError):
        check(lib.zmoe_layer_set_store(Lh._h, 0), "zmoe_layer_set_store")   # experts already loaded


def test_host_store_sm_tier_bit_identical_and_copies_a_third():
    # SMCACHE: misses outside the decoded cache keep their sign+mantissa planes
    # in HBM, so later misses copy only exponent blocks and indexes
    from zmoe.layer import MoELayer
    s = QWEN_SMALL
    L, w, wr, sg, sh = _build(s, 2, transient=2)
    layers = {}
    for sm in (0, 8):
        Lh = MoELayer(s, max_tokens=64, cache_slots=2, transient_slots=2, store="host", sm_slots=sm)
        Lh.set_router(wr, None, sg)
        Lh.set_shared(*sh)
        Lh.load_experts(w, num_file_chunks=3)
        layers[sm] = Lh
    per_miss = {}
    for i in range(5):
        x = syn.activations(24, s.hidden, seed=80 + i).cuda()
        want = L(x)
        for sm, Lh in layers.items():
            if i == 1:
                Lh.reset_stats()                        # planes admitted on the first forward; count from here
            assert torch.equal(want, Lh(x)), (i, sm)
    for sm, Lh in layers.items():
        Lh.sync()
        st = Lh.stats()
        assert st["decode_errors"] == 0 and st["misses"] > 0
        per_miss[sm] = st["host_copy_bytes"] / st["misses"]
    assert layers[8].stats()["sm_resident_tensors"] > 0 and layers[0].stats()["sm_resident_tensors"] == 0
    assert per_miss[8] < 0.45 * per_miss[0], per_miss


def test_engine_submit_host_pipeline_matches_device():
    # five steps with different inputs through the two staging slots; each
    # step's output lands in its own pinned buffer
    s = QWEN_SMALL
    L, *_ = _build(s, 2)
    xs = [syn.activations(16, s.hidden, seed=20 + i) for i in range(5)]
    want = [L(x.cuda()).cpu() for x in xs]
    xh = [x.pin_memory() for x in xs]
    oh = [torch.zeros_like(x).pin_memory() for x in xh]
    for a, b in zip(xh, oh):
        L.submit_host(a, b)
    L.join_host()
    torch.cuda.current_stream().synchronize()
    for w, o in zip(want, oh):
        assert torch.equal(w, o)
    # the synchronous call after pipelined steps still sees its own input
    o2 = torch.empty_like(xh[0]).pin_memory()
    L.forward_host(xh[0], o2)
    assert torch.equal(want[0], o2)


def test_engine_rejects_bad_inputs():
    from zmoe._lib import ZmoeError
    s = QWEN_SMALL
    L, *_ = _build(s, 2, T=8)
    with pytest.raises(ZmoeError):
        L(syn.activations(9, s.hidden).cuda())       # more tokens than max_tokens
