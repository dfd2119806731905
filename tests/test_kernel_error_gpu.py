"""Error path of the tcgen05 expert-FFN kernels: every mbarrier wait is
bounded, and a launch that gives one up drains its own copies, frees its TMEM,
returns, and raises an error word that the host reads.

The failure is made without faulting anything: the test hook
zmoe_debug_ffn_wait gives the next launches a short wait limit (about 10 ms)
and a TMA producer that issues no loads, so that the MMA warp's first wait
runs out.  The context stays usable, which the last call of each test checks by
running the same FFN again with the hook off."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import moe
from zmoe import synthetic as syn

pytestmark = pytest.mark.gpu
SHORT_WAIT = 20_000_000          # clock64 cycles, about 10 ms at 1.9 GHz


def _ffn_case(seed=5, H=512, I=192, rows=(3, 9, 40)):
    from zmoe import ops
    gen = torch.Generator().manual_seed(seed)
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    R = int(offs[-1])
    x = torch.randn(R, H, generator=gen).to(torch.bfloat16)
    mats = [[(torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16),
             (torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16),
             (torch.randn(H, I, generator=gen) * 0.05).to(torch.bfloat16)] for _ in rows]
    dev = [[t.cuda() for t in m] for m in mats]      # kept alive with the table that points at them
    wtab = ops.weight_table(dev, "cuda")
    return x, mats, (wtab, dev), offs


def _kernel_error(reset=1):
    from zmoe._lib import check, lib
    code = ctypes.c_int32(-1)
    check(lib.zmoe_kernel_error(ctypes.byref(code), reset), "zmoe_kernel_error")
    return code.value


def test_ffn_wait_timeout_is_reported_and_context_survives():
    from zmoe import ops
    from zmoe._lib import lib
    x, mats, (wtab, _dev), offs = _ffn_case()
    G, I = len(mats), mats[0][0].shape[0]
    _kernel_error(reset=1)
    assert _kernel_error() == 0
    lib.zmoe_debug_ffn_wait(SHORT_WAIT, 1)
    try:
        ops.expert_ffn(x.cuda(), wtab, torch.from_numpy(offs).cuda(), G, I, 0)
        torch.cuda.synchronize()
    finally:
        lib.zmoe_debug_ffn_wait(0, 0)
    assert _kernel_error(reset=1) == 1
    assert _kernel_error() == 0
    # same call with the hook off: correct result, no error
    y, _ = ops.expert_ffn(x.cuda(), wtab, torch.from_numpy(offs).cuda(), G, I, 0)
    torch.cuda.synchronize()
    assert _kernel_error() == 0
    ref = torch.cat([moe.swiglu_fp32(x[offs[g]:offs[g + 1]], *mats[g]) for g in range(G)])
    assert (y.float().cpu() - ref).abs().max().item() < 2e-2


def test_layer_reports_ffn_timeout_then_recovers():
    from zmoe._lib import ZmoeError, lib
    from zmoe.layer import MoELayer
    s = syn.LayerShape(hidden=256, num_experts=8, inter=64, topk=2, kind=0, shared_inter=128, shared_gate=True)
    w = syn.expert_weights(s, 1, std=0.05, seed=3)[0]
    wr, sg = syn.router_weights(s, std=0.05, seed=4)
    sh = syn.shared_weights(s, std=0.05, seed=5)
    L = MoELayer(s, max_tokens=32, cache_slots=4)
    L.set_router(wr, None, sg)
    L.set_shared(*sh)
    L.load_experts(w, num_file_chunks=3)
    x = syn.activations(24, s.hidden, seed=6)
    _kernel_error(reset=1)
    lib.zmoe_debug_ffn_wait(SHORT_WAIT, 1)
    try:
        L(x.cuda())
        with pytest.raises(ZmoeError, match="status 6"):
            L.sync()
    finally:
        lib.zmoe_debug_ffn_wait(0, 0)
    _kernel_error(reset=1)
    out = L(x.cuda())
    L.sync()
    ref, _ = moe.qwen_layer(x, wr, w, sh, sg, k=s.topk)
    assert (out.float().cpu() - ref.float()).abs().max().item() < 2e-2
    L.close()


def test_partial_weight_groups_are_rejected():
    from zmoe._lib import FfnArgs, lib
    x, mats, (wtab, _dev), offs = _ffn_case(rows=(4, 4))
    bad = wtab.clone()
    bad[3] = 0                     # group 1 without its gate matrix, down still set
    h = torch.empty(8, mats[0][0].shape[0], dtype=torch.bfloat16, device="cuda")
    y = torch.empty(8, x.shape[1], dtype=torch.float32, device="cuda")
    xd, od = x.cuda(), torch.from_numpy(offs).cuda()
    a = FfnArgs(xd.data_ptr(), bad.data_ptr(), od.data_ptr(), 2, 8, x.shape[1], mats[0][0].shape[0], 0,
                h.data_ptr(), y.data_ptr())
    assert lib.zmoe_expert_ffn(ctypes.byref(a), None) == 1
    assert b"only some of its weight pointers" in lib.zmoe_last_error()
