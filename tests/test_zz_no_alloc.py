"""zmoe_expert_ffn_noalloc: the FFN entry point for callers that cannot
allocate device memory (runtimes that own all device memory in their own pool,
or that must not call cudaMalloc/cudaFree mid-step) keeps its intermediate in a
file-scope device array.  Checked through the C ABI against zmoe_expert_ffn on
the same inputs, on two calls in a row (the array keeps the previous call's
contents, which must not leak into the next result).  Both entry points run
the same kernels on the same inputs, so the outputs must be bit-identical.

This file is collected last so that a run stopping at the first failure has
already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


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
    y = torch.full((R, H), float("nan"), dtype=torch.bfloat16, device="cuda")
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
        assert torch.equal(got, ref), call


def test_noalloc_qwen_shape_split_launch_bit_identical():
    # Qwen expert shape (H 2048, I 1408), 70 SwiGLU groups (two launches per
    # projection) with groups of more than 128 rows (several token tiles)
    from zmoe._lib import lib
    rows = [(g * 37) % 7 for g in range(70)]
    rows[3], rows[40], rows[69] = 300, 129, 256
    x, mats, wtab, offsets, G, R, H, I = _case(33, 0, rows, H=2048, I=1408)
    h = torch.empty(R, I, dtype=torch.bfloat16, device="cuda")
    ref = _call(lib.zmoe_expert_ffn, x, wtab, offsets, G, R, H, I, 0, h)
    for _ in range(2):
        got = _call(lib.zmoe_expert_ffn_noalloc, x, wtab, offsets, G, R, H, I, 0, None)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)


def test_noalloc_rejects_oversize_without_launching():
    from zmoe._lib import FfnArgs, lib
    dummy = torch.zeros(16, dtype=torch.int64, device="cuda")
    a = FfnArgs(dummy.data_ptr(), dummy.data_ptr(), None, 1, 1 << 20, 256, 64, 0, None, dummy.data_ptr())
    rc = lib.zmoe_expert_ffn_noalloc(ctypes.byref(a), None)
    assert rc == 3
    assert b"exceeds" in lib.zmoe_last_error()
