"""ORACLE — test infrastructure only: the reference's CPU path, timed as the
CPU baseline by bench.py (``cpu_baseline`` and ``--impl reference``).

Restates, with the reference's own libraries (liblz4 through ctypes, torch CPU
ops in BF16), what one MoE-layer forward costs the reference when experts are
stored exponent-compressed:

* every activated expert that is not in the decoded cache is decoded chunk by
  chunk on a thread pool: ``LZ4_decompress_safe_partial`` into a fresh buffer,
  then the bytes are copied into the staging plane
  (``csrc/tensor_engine/tensor_engine.cpp:421-474``,
  ``csrc/tensor_engine/compressors.cpp:195-211``), and the planes are
  recombined into BF16 (``csrc/kernels/tensor_recover.cu:25-30``; numpy here,
  the reference runs that step on the GPU);
* the block runs as ``customized/qwen.py:56-102`` does, with every expert
  computed by ``matmul(silu(x Wg^T) * (x Wu^T), Wd^T)`` in BF16
  (``csrc/dispatcher/expert_module.cpp:39-50``) and the combine accumulating
  into a BF16 buffer.
"""
from __future__ import annotations

import os
import time
from concurrent.futures import ThreadPoolExecutor
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch
import torch.nn.functional as F

from . import codec


def _decode_chunk(block, osz, exp, pos):
    exp[pos:pos + osz] = codec.lz4_decompress(block, osz)   # memcpy into the staging plane


def _recombine_into(exp, sm, out, a, b):
    s = sm[a:b].astype(np.uint16)
    out[a:b] = ((s >> 7) << 15) | (exp[a:b].astype(np.uint16) << 7) | (s & 0x7F)


def _decode_tensor(pool, blocks, osz, sm):
    exp = np.empty(sum(osz), np.uint8)
    futs, pos = [], 0
    for b, o in zip(blocks, osz):
        futs.append(pool.submit(_decode_chunk, b, o, exp, pos))
        pos += o
    for f in futs:
        f.result()
    smv = np.frombuffer(sm, np.uint8)
    bits = np.empty(exp.size, np.uint16)
    step = max(1, (exp.size + 7) // 8)
    rs = [pool.submit(_recombine_into, exp, smv, bits, a, min(exp.size, a + step)) for a in range(0, exp.size, step)]
    for f in rs:
        f.result()
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)


class ReferenceCPULayer:
    """One Qwen-style (SwiGLU + gated shared expert) layer on the CPU."""

    def __init__(self, shapes, encoded: Sequence[Sequence], w_router: torch.Tensor, bias: Optional[torch.Tensor],
                 w_shared_gate: Optional[torch.Tensor], shared: Optional[Sequence[torch.Tensor]], topk: int,
                 cache_experts: Sequence[int], threads: int = 0):
        self.shapes = shapes                     # per tensor (rows, cols)
        self.encoded = encoded                   # encoded[e][t] with .blocks .original_sizes .sm
        self.w_router = w_router.to(torch.bfloat16)
        self.bias = bias
        self.w_sg = w_shared_gate
        self.shared = shared
        self.topk = topk
        self.threads = threads or (os.cpu_count() or 1)
        self.pool = ThreadPoolExecutor(max_workers=self.threads)
        self.cache: Dict[int, List[torch.Tensor]] = {}
        for e in cache_experts:
            self.cache[e] = self._decode_expert(e)

    def close(self):
        self.pool.shutdown(wait=True)

    def _decode_expert(self, e: int) -> List[torch.Tensor]:
        out = []
        for t, enc in enumerate(self.encoded[e]):
            w = _decode_tensor(self.pool, enc.blocks, enc.original_sizes, enc.sm)
            out.append(w.view(*self.shapes[t]))
        return out

    def forward(self, x: torch.Tensor):
        """Returns (out, stats)."""
        t0 = time.perf_counter()
        logits = F.linear(x, self.w_router)                       # BF16 Linear
        if self.bias is not None:
            logits = (logits.float() + self.bias).to(torch.bfloat16)
        rw = F.softmax(logits, dim=1, dtype=torch.float)
        tw, ti = torch.topk(rw, self.topk, dim=-1)
        tw = tw.to(x.dtype)
        E = self.w_router.shape[0]
        counts = torch.bincount(ti.flatten(), minlength=E)
        active = [e for e in range(E) if counts[e] > 0]
        t1 = time.perf_counter()
        weights = {}
        misses = 0
        for e in active:
            if e in self.cache:
                weights[e] = self.cache[e]
            else:
                weights[e] = self._decode_expert(e)
                misses += 1
        t2 = time.perf_counter()
        out = torch.zeros_like(x)
        for e in active:
            tok, slot = (ti == e).nonzero(as_tuple=True)
            wg, wu, wd = weights[e]
            xe = x[tok]
            y = torch.matmul(F.silu(torch.matmul(xe, wg.t())) * torch.matmul(xe, wu.t()), wd.t())
            out[tok] += y * tw[tok, slot][:, None]
        if self.shared is not None:
            sg, su, sd = self.shared
            sh = torch.matmul(F.silu(torch.matmul(x, sg.t())) * torch.matmul(x, su.t()), sd.t())
            if self.w_sg is not None:
                sh = torch.sigmoid(F.linear(x, self.w_sg)) * sh
            out = out + sh
        t3 = time.perf_counter()
        return out, {"misses": misses, "active": len(active), "route_s": t1 - t0, "decode_s": t2 - t1,
                     "ffn_s": t3 - t2, "total_s": t3 - t0}
