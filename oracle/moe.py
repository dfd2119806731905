"""ORACLE — test infrastructure only (tests/, smoke(), bench.py's CPU legs).

CPU restatement of the reference's MoE-layer semantics on the hot path:

* Qwen1.5-MoE block   ``customized/qwen.py:44-102``
* DeepSeek-V2 block   ``customized/deepseek.py:67-116`` with the greedy gate
  ``models/deepseek/modeling_deepseek.py:424-476``
* Switch block        ``customized/switch_transformers.py:72-90`` with the
  transformers<4.47 ``SwitchTransformersTop1Router`` semantics (fp32 softmax,
  probabilities cast to the input dtype, argmax, cumsum capacity mask over the
  sequence axis, router_probs = max probability).
* Expert FFNs         ``csrc/dispatcher/expert_module.cpp:39-50`` (SwiGLU) and
  ``:67-78`` (ReLU).

Defined orders (the reference's own order is whatever cuBLAS/MKL pick):

* Router logits accumulate in fp32 in a fixed order: lane ``l`` of 32 sums
  ``x[h] * w[h]`` for ``h = 256*j + 8*l + i`` (j outer, i inner); the 32 lane
  sums are folded by an xor butterfly (16, 8, 4, 2, 1).  Products of two bf16
  values are exact in fp32, so fused and unfused multiply-add agree.
* Softmax uses ``exp_poly`` (Cody-Waite range reduction and a degree-7 Taylor
  polynomial, fp32, no fused multiply-add), the 32-lane strided sum + butterfly,
  and an IEEE division.  Everything is reproduced bit for bit by the kernel.
* Top-k: larger value first, ties to the lower expert index.
* Expert FFN accumulates in fp32; the SwiGLU intermediate and the expert
  output are each rounded to BF16 once (the reference's libtorch FFN returns
  BF16); the combine accumulates in fp32 and rounds the layer output once.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

F32 = np.float32


# --------------------------------------------------------------------------
# bf16 helpers
# --------------------------------------------------------------------------
def bf16_round(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, as torch .to(torch.bfloat16)."""
    t = torch.from_numpy(np.ascontiguousarray(a, dtype=F32))
    return t.to(torch.bfloat16).to(torch.float32).numpy()


def to_f32(t) -> np.ndarray:
    if isinstance(t, np.ndarray):
        return t.astype(F32, copy=False)
    return t.detach().to(torch.float32).cpu().numpy()


# --------------------------------------------------------------------------
# exp restatement shared with the router kernel
# --------------------------------------------------------------------------
_LOG2E = F32(1.4426950408889634)
# Cody-Waite split of ln 2: LN2_HI has 15 significant bits, so n*LN2_HI is
# exact for |n| <= 255.
_LN2_HI = F32(0.693145751953125)
_LN2_LO = F32(1.428606765330187e-06)
# 1/k! for k = 7..1, Horner order
_INV_FACT = [F32(1.0 / 5040.0), F32(1.0 / 720.0), F32(1.0 / 120.0), F32(1.0 / 24.0),
             F32(1.0 / 6.0), F32(0.5), F32(1.0)]


def exp_poly(x: np.ndarray) -> np.ndarray:
    """exp(x) for x <= 0 (softmax arguments), fp32, no fused multiply-add.

    Cody-Waite range reduction: n = rint(x log2 e), r = (x - n LN2_HI) - n LN2_LO
    with |r| <= 0.35; e^r by its Taylor series to degree 7 in Horner form
    (truncation below 6e-9); the result scaled by 2^n.  x below -87 returns 0.
    """
    x = np.asarray(x, dtype=F32)
    n = np.rint((x * _LOG2E).astype(F32)).astype(F32)
    r = (x - (n * _LN2_HI).astype(F32)).astype(F32)
    r = (r - (n * _LN2_LO).astype(F32)).astype(F32)
    p = np.full_like(r, _INV_FACT[0])
    for c in _INV_FACT[1:]:
        p = (p * r).astype(F32)
        p = (p + c).astype(F32)
    p = (p * r).astype(F32)
    p = (p + F32(1.0)).astype(F32)
    ni = n.astype(np.int32)
    out = np.ldexp(p, ni).astype(F32)
    return np.where(x < F32(-87.0), F32(0.0), out).astype(F32)


def _butterfly32(acc: np.ndarray) -> np.ndarray:
    """Fold the trailing axis of size 32 with an xor butterfly; returns [..., ]."""
    lanes = np.arange(32)
    for off in (16, 8, 4, 2, 1):
        acc = (acc + acc[..., lanes ^ off]).astype(F32)
    return acc[..., 0]


def router_logits(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """fp32 logits [T, E] of bf16-valued x [T, H] and w [E, H] in the defined order."""
    x = np.ascontiguousarray(x, dtype=F32)
    w = np.ascontiguousarray(w, dtype=F32)
    T, H = x.shape
    E = w.shape[0]
    if H % 256:
        raise ValueError("hidden size must be a multiple of 256")
    J = H // 256
    xr = x.reshape(T, J, 32, 8)
    wr = w.reshape(E, J, 32, 8)
    acc = np.zeros((T, E, 32), dtype=F32)
    for j in range(J):
        for i in range(8):
            prod = (xr[:, None, j, :, i] * wr[None, :, j, :, i]).astype(F32)   # exact
            acc = (acc + prod).astype(F32)
    return _butterfly32(acc)


def softmax_rows(logits: np.ndarray) -> np.ndarray:
    """Row softmax in the defined order: max, exp_poly, 32-lane strided sum, divide."""
    l = np.asarray(logits, dtype=F32)
    T, E = l.shape
    m = l.max(axis=1, keepdims=True)
    ex = exp_poly((l - m).astype(F32))
    E32 = (E + 31) // 32 * 32
    pad = np.zeros((T, E32), dtype=F32)
    pad[:, :E] = ex
    part = np.zeros((T, 32), dtype=F32)
    for j in range(E32 // 32):
        part = (part + pad[:, j * 32:(j + 1) * 32]).astype(F32)
    s = _butterfly32(part)[:, None]
    return (ex / s).astype(F32)


def topk_rule(values: np.ndarray, k: int):
    """Top-k per row: larger value first, ties to the lower index."""
    T, E = values.shape
    idx = np.empty((T, k), dtype=np.int32)
    val = np.empty((T, k), dtype=F32)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-float(values[t, e]), e))[:k]
        idx[t] = order
        val[t] = values[t, order]
    return idx, val


# --------------------------------------------------------------------------
# routers
# --------------------------------------------------------------------------
@dataclass
class Route:
    logits: np.ndarray            # [T, E] fp32 (bf16-valued for Qwen)
    probs: np.ndarray             # [T, E] fp32 softmax
    topk_idx: np.ndarray          # [T, k] int32, -1 = dropped (Switch over capacity)
    topk_w: np.ndarray            # [T, k] fp32 combine weights (bf16-valued for Qwen)
    counts: np.ndarray            # [E] int64 tokens per expert
    extra: dict = field(default_factory=dict)


def _counts(topk_idx: np.ndarray, E: int) -> np.ndarray:
    v = topk_idx[topk_idx >= 0]
    return np.bincount(v, minlength=E).astype(np.int64)


def route_qwen(x, w_gate, k: int, bias: Optional[np.ndarray] = None, norm_topk_prob=False) -> Route:
    """customized/qwen.py:44-54: bf16 Linear logits, fp32 softmax, topk, weights -> bf16."""
    l = router_logits(to_f32(x), to_f32(w_gate))
    if bias is not None:
        l = (l + np.asarray(bias, dtype=F32)[None, :]).astype(F32)
    l = bf16_round(l)
    p = softmax_rows(l)
    idx, val = topk_rule(p, k)
    if norm_topk_prob:
        val = (val / val.sum(axis=1, keepdims=True)).astype(F32)
    w = bf16_round(val)
    return Route(l, p, idx, w, _counts(idx, l.shape[1]))


def route_deepseek(x, w_gate, k: int, routed_scaling_factor: float = 1.0,
                   bias: Optional[np.ndarray] = None) -> Route:
    """modeling_deepseek.py:429-476 (greedy, norm_topk_prob=False): fp32 logits,
    softmax, topk(sorted=False) x routed_scaling_factor."""
    l = router_logits(to_f32(x), to_f32(w_gate))
    if bias is not None:
        l = (l + np.asarray(bias, dtype=F32)[None, :]).astype(F32)
    p = softmax_rows(l)
    idx, val = topk_rule(p, k)
    w = (val * F32(routed_scaling_factor)).astype(F32)
    return Route(l, p, idx, w, _counts(idx, l.shape[1]))


def route_switch(x, w_router, capacity: int, seq_len: int,
                 bias: Optional[np.ndarray] = None) -> Route:
    """transformers<4.47 SwitchTransformersTop1Router as used by
    customized/switch_transformers.py:72-90.  Tokens are [B, S] flattened with
    S = seq_len; capacity is counted per batch row along S."""
    l = router_logits(to_f32(x), to_f32(w_router))
    if bias is not None:
        l = (l + np.asarray(bias, dtype=F32)[None, :]).astype(F32)
    p = softmax_rows(l)
    pb = bf16_round(p)                               # .to(self.input_dtype)
    T, E = pb.shape
    arg = np.empty(T, dtype=np.int32)
    for t in range(T):
        arg[t] = int(np.flatnonzero(pb[t] == pb[t].max())[0])   # first maximal index
    rprob = pb.max(axis=1).astype(F32)
    idx = arg.copy()
    B = T // seq_len
    for b in range(B):
        seen = np.zeros(E, dtype=np.int64)
        for s in range(seq_len):
            t = b * seq_len + s
            seen[arg[t]] += 1
            if seen[arg[t]] > capacity:
                idx[t] = -1
    topk_idx = idx[:, None].astype(np.int32)
    topk_w = rprob[:, None].astype(F32)
    r = Route(l, p, topk_idx, topk_w, _counts(topk_idx, E))
    r.extra["argmax"] = arg
    return r


# --------------------------------------------------------------------------
# permute (token gather order of expert_dispatcher.cpp:326-330)
# --------------------------------------------------------------------------
def permute(topk_idx: np.ndarray, E: int):
    """Rows grouped by expert (ascending), tokens ascending inside each expert.

    Returns (offsets[E+1], token_of_row[R], row_of[T, k] with -1 for drops)."""
    T, k = topk_idx.shape
    counts = _counts(topk_idx, E)
    offsets = np.zeros(E + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    token_of_row = np.empty(int(offsets[-1]), dtype=np.int32)
    row_of = np.full((T, k), -1, dtype=np.int32)
    cursor = offsets[:-1].copy()
    for e in range(E):
        for t in range(T):
            for j in range(k):
                if topk_idx[t, j] == e:
                    r = cursor[e]
                    cursor[e] += 1
                    token_of_row[r] = t
                    row_of[t, j] = r
    return offsets, token_of_row, row_of


# --------------------------------------------------------------------------
# experts
# --------------------------------------------------------------------------
def swiglu_fp32(x: torch.Tensor, wg: torch.Tensor, wu: torch.Tensor, wd: torch.Tensor) -> torch.Tensor:
    """expert_module.cpp:39-50 with fp32 accumulation: the intermediate and the
    output are each rounded to BF16 once, as the reference's libtorch matmuls
    return them: y = bf16(bf16(silu(x Wg^T) * (x Wu^T)) Wd^T) (BF16 values, fp32 tensor)."""
    xf = x.float()
    g = xf @ wg.float().t()
    u = xf @ wu.float().t()
    h = (F.silu(g) * u).to(torch.bfloat16).float()
    return (h @ wd.float().t()).to(torch.bfloat16).float()


def relu_ffn_fp32(x: torch.Tensor, wi: torch.Tensor, wo: torch.Tensor) -> torch.Tensor:
    """expert_module.cpp:67-78: y = bf16(bf16(relu(x wi^T)) wo^T) (BF16 values, fp32 tensor)."""
    h = F.relu(x.float() @ wi.float().t()).to(torch.bfloat16).float()
    return (h @ wo.float().t()).to(torch.bfloat16).float()


def swiglu_bf16_ref(x, wg, wu, wd):
    """The reference's own rounding: every torch op returns BF16."""
    return torch.matmul(F.silu(torch.matmul(x, wg.t())) * torch.matmul(x, wu.t()), wd.t())


def relu_bf16_ref(x, wi, wo):
    return torch.matmul(F.relu(torch.matmul(x, wi.t())), wo.t())


# --------------------------------------------------------------------------
# whole layers (fp32 accumulate, one output rounding)
# --------------------------------------------------------------------------
def qwen_layer(x, w_gate, experts, shared, w_shared_gate, k=4, bias=None):
    """customized/qwen.py:56-102.  experts: list of (wg, wu, wd) bf16 tensors;
    shared: (wg, wu, wd); w_shared_gate: [1, H].  Returns (out bf16, Route, y rows)."""
    xb = x.to(torch.bfloat16)
    r = route_qwen(xb, w_gate, k, bias=bias)
    T, H = xb.shape
    out = torch.zeros(T, H, dtype=torch.float32)
    for e in range(len(experts)):
        tok = np.nonzero((r.topk_idx == e).any(axis=1))[0]
        if tok.size == 0:
            continue
        y = swiglu_fp32(xb[tok], *experts[e])
        wsel = torch.from_numpy(np.array([r.topk_w[t][list(r.topk_idx[t]).index(e)] for t in tok], dtype=F32))
        out[tok] += y * wsel[:, None]
    sh = swiglu_fp32(xb, *shared)
    sg_logit = torch.from_numpy(router_logits(to_f32(xb), to_f32(w_shared_gate)))   # [T, 1]
    sg = torch.sigmoid(sg_logit.to(torch.bfloat16).float())
    out = out + sg * sh
    return out.to(torch.bfloat16), r


def qwen_layer_bf16(x, w_gate, experts, shared, w_shared_gate, k=4, bias=None, topk_idx=None, topk_w=None):
    """customized/qwen.py:56-102 with the reference's own roundings: every
    torch op in BF16 (expert_module.cpp:39-50 via swiglu_bf16_ref), the routed
    outputs scaled by BF16 weights and added into a BF16 buffer in ascending
    expert order (qwen.py:89-93), the shared expert scaled by a BF16 sigmoid
    gate and added last (qwen.py:98-100).  topk_idx / topk_w, when given,
    replace this module's routing (to replay a selection made elsewhere, e.g.
    where the reference broke an exact tie differently).  Returns BF16 [T, H]."""
    xb = x.to(torch.bfloat16)
    r = route_qwen(xb, w_gate, k, bias=bias)
    idx = r.topk_idx if topk_idx is None else np.asarray(topk_idx)
    tw = torch.from_numpy(r.topk_w if topk_w is None else np.asarray(topk_w, dtype=F32)).to(torch.bfloat16)
    T, H = xb.shape
    out = torch.zeros(T, H, dtype=torch.bfloat16)
    for e in range(len(experts)):
        tok = np.nonzero((idx == e).any(axis=1))[0]
        if tok.size == 0:
            continue
        y = swiglu_bf16_ref(xb[tok], *experts[e])
        wsel = torch.stack([tw[t][list(idx[t]).index(e)] for t in tok])
        out[tok] += y * wsel[:, None]
    sh = swiglu_bf16_ref(xb, *shared)
    return out + torch.sigmoid(F.linear(xb, w_shared_gate.to(torch.bfloat16))) * sh


def deepseek_layer(x, w_gate, experts, shared, k=6, routed_scaling_factor=1.0, bias=None):
    """customized/deepseek.py:67-116 (shared experts added without a gate)."""
    xb = x.to(torch.bfloat16)
    r = route_deepseek(xb, w_gate, k, routed_scaling_factor, bias=bias)
    T, H = xb.shape
    out = torch.zeros(T, H, dtype=torch.float32)
    for e in range(len(experts)):
        tok = np.nonzero((r.topk_idx == e).any(axis=1))[0]
        if tok.size == 0:
            continue
        y = swiglu_fp32(xb[tok], *experts[e])
        wsel = torch.from_numpy(np.array([r.topk_w[t][list(r.topk_idx[t]).index(e)] for t in tok], dtype=F32))
        out[tok] += y * wsel[:, None]
    if shared is not None:
        out = out + swiglu_fp32(xb, *shared)
    return out.to(torch.bfloat16), r


def switch_layer(x, w_router, experts, capacity, seq_len, bias=None):
    """customized/switch_transformers.py:72-90: accepted tokens take the expert
    output, dropped ones keep their input; both are scaled by router_probs."""
    xb = x.to(torch.bfloat16)
    r = route_switch(xb, w_router, capacity, seq_len, bias=bias)
    nxt = xb.float().clone()
    for e in range(len(experts)):
        tok = np.nonzero(r.topk_idx[:, 0] == e)[0]
        if tok.size == 0:
            continue
        nxt[tok] = relu_ffn_fp32(xb[tok], *experts[e])
    out = torch.from_numpy(r.topk_w[:, 0:1]) * nxt
    return out.to(torch.bfloat16), r
