"""Expert-parallel MoE layer: experts sharded over the ranks of a process group.

Placement: rank r owns the contiguous expert block [r*E//P, (r+1)*E//P) (E = 60
over 8 ranks gives 7 or 8 experts each).  Router, shared expert and tokens are
data-parallel: every rank routes its own tokens with the replicated router.

One forward on every rank:

1. router + permute of the local tokens (rows grouped by global expert, so the
   rows bound for one rank are contiguous);
2. all-to-all of the per-expert row counts (int32, E on each side);
3. all-to-all of the permuted BF16 rows (sizes from the counts);
4. regroup the received rows by local expert (a row gather);
5. the expert stage of the local engine (cache decision, miss decode on the
   GPU, tcgen05 grouped FFN) -> BF16 rows;
6. inverse regroup, all-to-all of the BF16 rows back to their token's rank;
7. shared expert and gate-weighted combine on the local tokens.

This is the exchange the reference's vendored DeepSeek expert parallelism and
its dispatcher imply (``experts/expert_executor.py:40-84`` drives one rank's
experts; ``csrc/dispatcher/expert_dispatcher.cpp:326-330`` gathers an expert's
rows).  Two implementations: :class:`NativeEPLayer` runs the whole forward in
libzmoe.so (zmoe_ep_forward, NCCL point-to-point calls on the group's own
communicator, one host wait per forward); :class:`EPMoELayer` runs the same
steps in Python over ``torch.distributed`` with the arithmetic behind an
object (``EPKernels`` on a GPU, or the oracle's kernels on the CPU for gloo
tests).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np
import torch
import torch.distributed as dist

from .synthetic import LayerShape


class ExpertPartition:
    """Contiguous, balanced expert blocks: rank r owns [bounds[r], bounds[r+1])."""

    def __init__(self, num_experts: int, world: int):
        if world < 1 or num_experts < world:
            raise ValueError(f"cannot shard {num_experts} experts over {world} ranks")
        self.E, self.P = num_experts, world
        self.bounds = [r * num_experts // world for r in range(world + 1)]

    def owned(self, rank: int) -> range:
        return range(self.bounds[rank], self.bounds[rank + 1])

    def sizes(self) -> List[int]:
        return [self.bounds[r + 1] - self.bounds[r] for r in range(self.P)]

    def owner(self, expert: int) -> int:
        for r in range(self.P):
            if expert < self.bounds[r + 1]:
                return r
        raise ValueError(f"expert {expert} outside [0, {self.E})")


def regroup_plan(recv_counts: np.ndarray):
    """Rows received as [source rank][local expert] -> [local expert][source rank].

    recv_counts: int [P, E_local].  Returns (index, inverse, counts_local) where
    grouped[i] = received[index[i]] and received[j] = grouped[inverse[j]]."""
    recv_counts = np.asarray(recv_counts, dtype=np.int64)
    P, El = recv_counts.shape
    flat = recv_counts.reshape(-1)
    start = np.zeros(flat.size, dtype=np.int64)                 # start of block (src, e) in received order
    if flat.size:
        start[1:] = np.cumsum(flat)[:-1]
    start = start.reshape(P, El)
    parts = [np.arange(start[s, e], start[s, e] + recv_counts[s, e], dtype=np.int64)
             for e in range(El) for s in range(P)]
    index = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
    inverse = np.empty_like(index)
    inverse[index] = np.arange(index.size, dtype=np.int64)
    return index.astype(np.int32), inverse.astype(np.int32), recv_counts.sum(axis=0).astype(np.int32)


class EPKernels:
    """The GPU arithmetic of one rank, through the C ABI (zmoe.ops / MoELayer)."""

    def __init__(self, shape: LayerShape, w_router: torch.Tensor, bias: Optional[torch.Tensor],
                 w_shared_gate: Optional[torch.Tensor], shared: Optional[Sequence[torch.Tensor]], device):
        from . import ops
        self.ops = ops
        self.s = shape
        dev = torch.device(device)
        self.w = w_router.to(torch.bfloat16).contiguous().to(dev)
        self.bias = bias.to(torch.float32).contiguous().to(dev) if bias is not None else None
        self.wsg = w_shared_gate.to(torch.bfloat16).contiguous().to(dev) if w_shared_gate is not None else None
        self.shared = [t.to(torch.bfloat16).contiguous().to(dev) for t in shared] if shared else None
        self.shared_tab = ops.weight_table([self.shared]) if self.shared else None
        self.mode = ops.ROUTE_SWITCH if shape.kind == 1 else (ops.ROUTE_QWEN if shape.shared_gate else ops.ROUTE_DEEPSEEK)

    def route(self, x):
        _, idx, tw, sg = self.ops.router(x, self.w, self.s.topk, self.mode, self.bias, self.wsg, self.s.scaling,
                                         want_logits=False)
        cap = self.s.capacity if self.s.kind == 1 else 0
        counts, _, row_of, _, xp = self.ops.permute(idx, x, self.s.num_experts, cap,
                                                    self.s.seq_len if cap else 0)
        return counts, row_of, tw, sg, xp

    def gather_rows(self, src: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
        out = torch.empty((index.numel(),) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
        row_bytes = src[0].numel() * src.element_size() if src.shape[0] else 16
        self.ops.check(self.ops.lib.zmoe_gather_rows(src.data_ptr(), index.data_ptr(), index.numel(), row_bytes,
                                                     out.data_ptr(), self.ops._stream()), "zmoe_gather_rows")
        return out

    def shared_expert(self, x):
        if self.shared is None:
            return None
        y, _ = self.ops.expert_ffn(x, self.shared_tab, None, 1, self.s.shared_inter, 0)
        return y

    def combine(self, y, row_of, tw, sg, y_shared, x):
        return self.ops.combine(y, row_of, tw, self.mode, y_shared, sg, x)


class EPMoELayer:
    """One rank's share of an expert-parallel MoE layer.

    ``local`` runs the expert stage for this rank's experts (an object with
    ``experts(x_rows, counts) -> y_rows``; by default a :class:`MoELayer` over
    the owned experts); ``kernels`` does routing, gathers, shared expert and
    combine (by default :class:`EPKernels` on this rank's GPU)."""

    def __init__(self, shape: LayerShape, kernels, local, group=None):
        self.s = shape
        self.group = group
        self.P = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.part = ExpertPartition(shape.num_experts, self.P)
        self.mine = self.part.owned(self.rank)
        self.K = kernels
        self.local = local

    @staticmethod
    def local_shape(shape: LayerShape, n_local: int) -> LayerShape:
        return LayerShape(shape.hidden, n_local, shape.inter, shape.topk, shape.kind, 0, False, shape.scaling,
                          shape.capacity, shape.seq_len, 0.0)

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: List[int], in_splits: List[int]):
        if self.P == 1:
            out.copy_(inp)
            return
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        s, P, El = self.s, self.P, len(self.mine)
        H = s.hidden
        counts, row_of, tw, sg, xp = self.K.route(x)
        # the shared expert needs only x: on a side stream it overlaps the exchange
        side = None
        if x.is_cuda:
            if getattr(self, "_side", None) is None:
                self._side = torch.cuda.Stream(device=x.device)
            side = self._side
            side.wait_stream(torch.cuda.current_stream(x.device))
            with torch.cuda.stream(side):
                y_sh = self.K.shared_expert(x)
        else:
            y_sh = self.K.shared_expert(x)
        # 1. counts: rows for expert e of rank r go to r
        recv_counts = torch.empty(P * El, dtype=torch.int32, device=x.device)
        self._a2a(recv_counts, counts, [El] * P, self.part.sizes())
        both = torch.cat([counts.to(torch.int32), recv_counts]).cpu().numpy().astype(np.int64)
        c_send, c_recv = both[:s.num_experts], both[s.num_experts:].reshape(P, El)
        send_rows = [int(c_send[self.part.bounds[r]:self.part.bounds[r + 1]].sum()) for r in range(P)]
        recv_rows = [int(v) for v in c_recv.sum(axis=1)]
        n_send, n_recv = sum(send_rows), sum(recv_rows)
        # 2. rows out
        recv_x = torch.empty(n_recv, H, dtype=x.dtype, device=x.device)
        self._a2a(recv_x, xp[:n_send], recv_rows, send_rows)
        # 3. local experts on rows grouped by expert
        index, inverse, counts_local = regroup_plan(c_recv)
        idx_dev = torch.from_numpy(np.concatenate([index, inverse])).to(x.device, non_blocking=True)
        xg = self.K.gather_rows(recv_x, idx_dev[:n_recv]) if n_recv else recv_x
        yg = self.local.experts(xg, counts_local)
        y_src = self.K.gather_rows(yg, idx_dev[n_recv:]) if n_recv else yg
        # 4. rows back, in the order they left
        y_back = torch.empty(n_send, H, dtype=y_src.dtype, device=x.device)
        self._a2a(y_back, y_src, send_rows, recv_rows)
        # 5. combine with the shared expert on the local tokens
        if side is not None:
            torch.cuda.current_stream(x.device).wait_stream(side)
            if y_sh is not None:
                y_sh.record_stream(torch.cuda.current_stream(x.device))
        if n_send == 0:                                   # every token dropped (Switch capacity)
            y_back = torch.zeros(1, H, dtype=y_src.dtype, device=x.device)
        return self.K.combine(y_back, row_of, tw, sg, y_sh, x)

    __call__ = forward


def nccl_comm_ptr(device: int, group=None) -> int:
    """The ncclComm_t (as an integer) of a torch.distributed NCCL group on
    this rank's GPU; a barrier first makes sure the communicator exists."""
    pg = group if group is not None else dist.distributed_c10d._get_default_group()
    dist.barrier(group=pg)
    return int(pg._get_backend(torch.device("cuda", device))._comm_ptr())


class NativeEPLayer:
    """One rank's share of an expert-parallel MoE layer, run by libzmoe.so
    (zmoe_ep_forward): routing, NCCL exchanges of counts and BF16 rows, the
    local engine's expert stage and the combine, in C++ with one host wait per
    forward.  ``local`` is the :class:`MoELayer` holding this rank's experts."""

    def __init__(self, shape: LayerShape, local, w_router, bias, w_shared_gate, shared, max_tokens: int,
                 device: int, group=None):
        import ctypes
        from ._lib import EPConfig, LayerConfig, check, lib
        from .layer import route_mode
        self.s, self.local, self.engine = shape, local, local
        self.P = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = torch.device("cuda", device)
        comm = nccl_comm_ptr(device, group) if self.P > 1 else None
        lc = LayerConfig(shape.hidden, shape.num_experts, shape.inter, shape.topk, shape.kind, route_mode(shape), 0,
                         shape.scaling, shape.shared_inter, shape.capacity, shape.seq_len, max_tokens, 0, 0, 0, 0.0, 0)
        cfg = EPConfig(lc, self.rank, self.P, comm)
        h = ctypes.c_void_p()
        check(lib.zmoe_ep_create(ctypes.byref(cfg), local._h, ctypes.byref(h)), "zmoe_ep_create")
        self._h, self._lib, self._check = h, lib, check
        host = lambda t: None if t is None else t.detach().contiguous().cpu()
        self._keep = [host(w_router.to(torch.bfloat16)), host(bias.to(torch.float32)) if bias is not None else None,
                      host(w_shared_gate.to(torch.bfloat16)) if w_shared_gate is not None else None]
        ptr = lambda t: None if t is None else t.data_ptr()
        check(lib.zmoe_ep_set_router(h, *[ptr(t) for t in self._keep]), "zmoe_ep_set_router")
        if shared is not None:
            sh = [host(t.to(torch.bfloat16)) for t in shared]
            check(lib.zmoe_ep_set_shared(h, *[t.data_ptr() for t in sh]), "zmoe_ep_set_shared")
        self.max_tokens = max_tokens

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("x must be a contiguous CUDA BF16 tensor")
        if out is None:
            out = torch.empty_like(x)
        self._check(self._lib.zmoe_ep_forward(self._h, x.data_ptr(), x.shape[0], out.data_ptr(),
                                              torch.cuda.current_stream(self.device).cuda_stream), "zmoe_ep_forward")
        return out

    __call__ = forward

    def close(self):
        if getattr(self, "_h", None):
            self._lib.zmoe_ep_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def build_gpu_layer(shape: LayerShape, experts_encoded, w_router, bias, w_shared_gate, shared, max_tokens: int,
                    cache_slots: int, device: int, group=None, warm: Sequence[int] = (), native: bool = True):
    """This rank's share of an expert-parallel layer on its GPU.
    experts_encoded[e] = encoded tensors of global expert e (EncodedTensor;
    None for experts other ranks own); only the owned experts are loaded.
    max_tokens bounds the tokens of one rank; warm = global expert ids to
    decode into the cache up front (those this rank owns).  native: the C++
    layer (NativeEPLayer, NCCL from libzmoe.so); otherwise the Python
    exchange (EPMoELayer over torch.distributed)."""
    from .layer import MoELayer
    P = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    part = ExpertPartition(shape.num_experts, P)
    mine = part.owned(rank)
    ls = EPMoELayer.local_shape(shape, len(mine))
    local = MoELayer(ls, max_tokens=P * max_tokens, cache_slots=min(cache_slots, len(mine)), device=device)
    for j, e in enumerate(mine):
        for t, enc in enumerate(experts_encoded[e]):
            local.load_encoded(j, t, enc)
    w = [e - mine.start for e in warm if e in mine]
    if w:
        local.warm_cache(w[:local_cache_cap(cache_slots, len(mine))])
    if native:
        return NativeEPLayer(shape, local, w_router, bias, w_shared_gate, shared, max_tokens, device, group)
    kern = EPKernels(shape, w_router, bias, w_shared_gate, shared, torch.device("cuda", device))
    layer = EPMoELayer(shape, kern, local, group)
    layer.engine = local
    return layer


def local_cache_cap(cache_slots: int, n_local: int) -> int:
    return max(0, min(cache_slots, n_local))
