"""Test helper: the arithmetic of one expert-parallel rank restated on the CPU
with the oracle (routing, permute, FFNs, combine), so the exchange logic of
``zmoe.ep.EPMoELayer`` runs under gloo without a GPU.  Test infrastructure only."""
from __future__ import annotations

import numpy as np
import torch

from oracle import moe


class OracleKernels:
    def __init__(self, s, w_router, bias, w_shared_gate, shared):
        self.s, self.w, self.bias, self.wsg, self.shared = s, w_router, bias, w_shared_gate, shared

    def route(self, x):
        s = self.s
        b = None if self.bias is None else self.bias.numpy()
        if s.kind == 1:
            r = moe.route_switch(x, self.w, s.capacity, s.seq_len, bias=b)
        elif s.shared_gate:
            r = moe.route_qwen(x, self.w, s.topk, bias=b)
        else:
            r = moe.route_deepseek(x, self.w, s.topk, s.scaling, bias=b)
        _, tor, row_of = moe.permute(r.topk_idx, s.num_experts)
        counts = torch.from_numpy(r.counts.astype(np.int32))
        xp = x[torch.from_numpy(tor).long()]
        sg = None
        if s.shared_gate:
            lg = torch.from_numpy(moe.router_logits(moe.to_f32(x), moe.to_f32(self.wsg)))
            sg = torch.sigmoid(lg.to(torch.bfloat16).float())[:, 0]
        return counts, torch.from_numpy(row_of), torch.from_numpy(r.topk_w), sg, xp

    def gather_rows(self, src, index):
        return src[index.long()].contiguous()

    def shared_expert(self, x):
        return None if self.shared is None else moe.swiglu_fp32(x, *self.shared)

    def combine(self, y, row_of, tw, sg, y_shared, x):
        T, k = row_of.shape
        out = torch.zeros(T, x.shape[1], dtype=torch.float32)
        for t in range(T):
            for j in range(k):
                r = int(row_of[t, j])
                if self.s.kind == 1:
                    out[t] += float(tw[t, j]) * (y[r] if r >= 0 else x[t].float())
                elif r >= 0:
                    out[t] += float(tw[t, j]) * y[r]
        if y_shared is not None:
            out += (sg[:, None] * y_shared) if sg is not None else y_shared
        return out.to(torch.bfloat16)


class OracleLocalExperts:
    """Expert stage of one rank: weights of its own experts, in order."""

    def __init__(self, s, weights):
        self.s, self.weights = s, weights

    def experts(self, x_rows, counts):
        out = torch.empty(int(np.sum(counts)), self.s.hidden, dtype=torch.float32)
        r = 0
        for e, c in enumerate(counts):
            c = int(c)
            if c:
                f = moe.relu_ffn_fp32 if self.s.kind == 1 else moe.swiglu_fp32
                out[r:r + c] = f(x_rows[r:r + c], *self.weights[e])
            r += c
        return out
