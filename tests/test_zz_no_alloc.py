"""zmoe_expert_ffn_noalloc: the FFN entry point for callers that cannot
allocate device memory (runtimes that own all device memory in their own pool,
or that must not call cudaMalloc/cudaFree mid-step) keeps its intermediate in a
file-scope device array.  Checked through the C ABI against zmoe_expert_ffn on
the same inputs, on two calls in a row (the array keeps the previous call's
contents, which must not leak into the next result).

This file is collected last so that a run stopping at the first failure has
already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL_MAX_ABS = 2e-2
TOL_MEAN_REL = 5e-3


def _close(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    d = np.abs(a - b)
    return d.max(), d.mean() / max(np.abs(b).mean(), 1e-12)


def _case(seed, kind, rows, H=512, I=320):
    from zmoe import ops
    gen = torch.Generator().manual_seed(seed)
    G = len(rows)
    offs = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    R = int(offs[-1])
    x = torch.randn(R, H, generator=gen).to(torch.bfloat16).cuda()
    mats = []
    for _ in range(G):
        up = (torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16).cuda() if kind == 0 else None
        mats.append([(torch.randn(I, H, generator=gen) * 0.05).to(torch.bfloat16).cuda(), up,
                     (torch.randn(H, I, generator=gen) * 0.05).to(torch.bfloat16).cuda()])
    wtab = ops.weight_table(mats, "cuda")
    return x, mats, wtab, torch.from_numpy(offs).cuda(), G, R, H, I


def _call(fn, x, wtab, offsets, G, R, H, I, kind, h):
    from zmoe._lib import FfnArgs, check
    y = torch.full((R, H), float("nan"), dtype=torch.float32, device="cuda")
    a = FfnArgs(x.data_ptr(), wtab.data_ptr(), offsets.data_ptr(), G, R, H, I, kind,
                h.data_ptr() if h is not None else None, y.data_ptr())
    check(fn(ctypes.byref(a), torch.cuda.current_stream().cuda_stream), fn.__name__)
    return y


def test_noalloc_matches_allocating_entry_point_twice():
    from zmoe._lib import lib
    for call, (seed, kind, rows) in enumerate([(31, 0, [5, 0, 17, 40]), (32, 1, [3, 64, 1])]):
        x, mats, wtab, offsets, G, R, H, I = _case(seed, kind, rows)
        h = torch.empty(R, I, dtype=torch.bfloat16, device="cuda")
        ref = _call(lib.zmoe_expert_ffn, x, wtab, offsets, G, R, H, I, kind, h)
        got = _call(lib.zmoe_expert_ffn_noalloc, x, wtab, offsets, G, R, H, I, kind, None)
        torch.cuda.synchronize()
        assert not torch.isnan(got).any(), call
        mx, mr = _close(got.cpu().numpy(), ref.cpu().numpy())
        assert mx <= TOL_MAX_ABS and mr <= TOL_MEAN_REL, (call, mx, mr)


def test_noalloc_rejects_oversize_without_launching():
    from zmoe._lib import FfnArgs, lib
    dummy = torch.zeros(16, dtype=torch.int64, device="cuda")
    a = FfnArgs(dummy.data_ptr(), dummy.data_ptr(), None, 1, 1 << 20, 256, 64, 0, None, dummy.data_ptr())
    rc = lib.zmoe_expert_ffn_noalloc(ctypes.byref(a), None)
    assert rc == 3
    assert b"exceeds" in lib.zmoe_last_error()
