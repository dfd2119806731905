"""``MoELayer``: Python handle over the C++ layer engine of libzmoe.so.

The engine keeps every routed expert compressed in HBM (LZ4 exponent chunks +
raw sign+mantissa plane, the reference's storage form), keeps ``cache_slots``
decoded experts resident, and decodes misses on the GPU inside
``forward``.  See include/zmoe.h (zmoe_layer_*).
"""
from __future__ import annotations

import ctypes
from typing import Iterable, List, Optional, Sequence

import torch

from . import codec as zcodec
from ._lib import LayerConfig, LayerStats, check, lib
from .synthetic import LayerShape

POLICIES = {"ZipMoE": 0, "LFU": 1, "LRU": 2, "FIFO": 3}
STORES = {"device": 0, "host": 1}


def route_mode(s: LayerShape) -> int:
    if s.kind == 1:
        return 2
    return 0 if s.shared_gate else 1


class MoELayer:
    def __init__(self, shape: LayerShape, max_tokens: int, cache_slots: int, transient_slots: int = 0,
                 policy: str = "ZipMoE", state_margin: float = 0.1, device: int = 0, store: str = "device",
                 sm_slots: int = 0):
        self.shape = shape
        self.device = torch.device("cuda", device)
        torch.cuda.set_device(self.device)
        cfg = LayerConfig(shape.hidden, shape.num_experts, shape.inter, shape.topk, shape.kind, route_mode(shape),
                          0, shape.scaling, shape.shared_inter, shape.capacity, shape.seq_len, max_tokens,
                          cache_slots, transient_slots, POLICIES[policy], state_margin, sm_slots)
        h = ctypes.c_void_p()
        check(lib.zmoe_layer_create(ctypes.byref(cfg), ctypes.byref(h)), "zmoe_layer_create")
        self._h = h
        if store not in STORES:
            raise ValueError(f"store must be one of {sorted(STORES)}")
        # "host": compressed experts in pinned host memory, copied in per miss;
        # sm_slots: how many experts' sign+mantissa planes the host tier keeps in HBM
        check(lib.zmoe_layer_set_store(h, STORES[store]), "zmoe_layer_set_store")
        self.max_tokens = max_tokens

    def close(self):
        if getattr(self, "_h", None):
            lib.zmoe_layer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @staticmethod
    def _host(t: Optional[torch.Tensor]):
        return None if t is None else t.detach().contiguous().cpu()

    def set_router(self, w_router: torch.Tensor, bias: Optional[torch.Tensor] = None,
                   w_shared_gate: Optional[torch.Tensor] = None):
        w = self._host(w_router.to(torch.bfloat16))
        b = self._host(bias.to(torch.float32)) if bias is not None else None
        g = self._host(w_shared_gate.to(torch.bfloat16)) if w_shared_gate is not None else None
        self._keep = (w, b, g)
        check(lib.zmoe_layer_set_router(self._h, w.data_ptr(), b.data_ptr() if b is not None else None,
                                        g.data_ptr() if g is not None else None), "zmoe_layer_set_router")

    def set_shared(self, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor):
        ts = [self._host(t.to(torch.bfloat16)) for t in (gate, up, down)]
        check(lib.zmoe_layer_set_shared(self._h, *[t.data_ptr() for t in ts]), "zmoe_layer_set_shared")

    def load_encoded(self, expert: int, tensor: int, enc: zcodec.EncodedTensor):
        n = len(enc.blocks)
        bufs = [ctypes.create_string_buffer(b, len(b)) for b in enc.blocks]
        ptrs = (ctypes.c_void_p * n)(*[ctypes.addressof(b) for b in bufs])
        sizes = (ctypes.c_uint32 * n)(*[len(b) for b in enc.blocks])
        osz = (ctypes.c_uint32 * n)(*enc.original_sizes)
        sm = ctypes.create_string_buffer(enc.sm, len(enc.sm))
        check(lib.zmoe_layer_load_expert(self._h, expert, tensor, ptrs, sizes, osz, n, ctypes.addressof(sm),
                                         enc.numel), "zmoe_layer_load_expert")

    def load_experts(self, experts: Sequence[Sequence[torch.Tensor]], num_file_chunks: int = 3,
                     codec: str = "LZ4HC", level: int = 9, threads: int = 0) -> List[List[zcodec.EncodedTensor]]:
        """Encode and load every expert; experts[e] = [gate, up, down] or [wi, wo]."""
        flat = [t for e in experts for t in e]
        enc = zcodec.encode_tensors(flat, num_file_chunks, codec, level, threads)
        per = len(experts[0])
        out = []
        for e in range(len(experts)):
            row = enc[e * per:(e + 1) * per]
            for t, et in enumerate(row):
                self.load_encoded(e, t, et)
            out.append(row)
        return out

    def warm_cache(self, experts: Iterable[int]):
        ex = list(experts)
        arr = (ctypes.c_int * max(len(ex), 1))(*ex)
        check(lib.zmoe_layer_warm_cache(self._h, arr, len(ex), torch.cuda.current_stream(self.device).cuda_stream),
              "zmoe_layer_warm_cache")

    def prefetch(self, experts: Iterable[int]):
        """Decode experts into cache slots ahead of use (zmoe_layer_prefetch),
        on the layer's decode stream after the work already queued on the
        current stream; returns without waiting."""
        ex = list(experts)
        arr = (ctypes.c_int * max(len(ex), 1))(*ex)
        check(lib.zmoe_layer_prefetch(self._h, arr, len(ex), torch.cuda.current_stream(self.device).cuda_stream),
              "zmoe_layer_prefetch")

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise ValueError("x must be a contiguous CUDA BF16 tensor")
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        check(lib.zmoe_layer_forward(self._h, x.data_ptr(), T, out.data_ptr(),
                                     torch.cuda.current_stream(self.device).cuda_stream), "zmoe_layer_forward")
        return out

    __call__ = forward

    def forward_host(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Host BF16 in, host BF16 out (pinned for full speed)."""
        check(lib.zmoe_layer_forward_host(self._h, x.data_ptr(), x.shape[0], out.data_ptr(),
                                          torch.cuda.current_stream(self.device).cuda_stream),
              "zmoe_layer_forward_host")
        return out

    def submit_host(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Pipelined forward_host (zmoe_layer_submit_host): returns once the step
        is queued; out is written after join_host() and a wait on the stream.
        x and out must be pinned host BF16 [T, H] and stay untouched until then."""
        check(lib.zmoe_layer_submit_host(self._h, x.data_ptr(), x.shape[0], out.data_ptr(),
                                         torch.cuda.current_stream(self.device).cuda_stream),
              "zmoe_layer_submit_host")
        return out

    def join_host(self):
        """The current stream waits for every submitted step's output copy."""
        check(lib.zmoe_layer_join_host(self._h, torch.cuda.current_stream(self.device).cuda_stream),
              "zmoe_layer_join_host")

    def experts(self, x_rows: torch.Tensor, counts, y: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Expert stage alone (zmoe_layer_experts): x_rows [rows, H] BF16 grouped
        by this layer's experts, counts[e] rows of expert e; returns BF16 [rows, H]."""
        import numpy as np
        c = np.ascontiguousarray(np.asarray(counts, dtype=np.int32))
        if c.size != self.shape.num_experts:
            raise ValueError(f"counts has {c.size} entries, layer has {self.shape.num_experts} experts")
        rows = int(c.sum())
        if rows and (not x_rows.is_cuda or x_rows.dtype != torch.bfloat16 or not x_rows.is_contiguous()
                     or x_rows.shape[0] < rows):
            raise ValueError("x_rows must be a contiguous CUDA BF16 tensor with sum(counts) rows")
        if y is None:
            y = torch.empty(rows, self.shape.hidden, dtype=torch.bfloat16, device=self.device)
        check(lib.zmoe_layer_experts(self._h, x_rows.data_ptr() if rows else None,
                                     c.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), rows,
                                     y.data_ptr() if rows else None,
                                     torch.cuda.current_stream(self.device).cuda_stream), "zmoe_layer_experts")
        return y

    def sync(self):
        check(lib.zmoe_layer_sync(self._h, torch.cuda.current_stream(self.device).cuda_stream), "zmoe_layer_sync")

    def stats(self) -> dict:
        s = LayerStats()
        check(lib.zmoe_layer_get_stats(self._h, ctypes.byref(s)), "zmoe_layer_get_stats")
        return {n: getattr(s, n) for n, _ in LayerStats._fields_}

    def reset_stats(self):
        check(lib.zmoe_layer_reset_stats(self._h), "zmoe_layer_reset_stats")

    def set_timing(self, on: bool = True):
        check(lib.zmoe_layer_set_timing(self._h, int(on)), "zmoe_layer_set_timing")

    def last_counts(self) -> List[int]:
        """Tokens per expert in the last forward (zmoe_layer_last_counts)."""
        n = ctypes.c_int()
        buf = (ctypes.c_int32 * self.shape.num_experts)()
        check(lib.zmoe_layer_last_counts(self._h, buf, self.shape.num_experts, ctypes.byref(n)),
              "zmoe_layer_last_counts")
        return [int(buf[i]) for i in range(n.value)]

    def cached_experts(self) -> List[int]:
        n = ctypes.c_int()
        buf = (ctypes.c_int32 * self.shape.num_experts)()
        check(lib.zmoe_layer_cached_experts(self._h, buf, self.shape.num_experts, ctypes.byref(n)),
              "zmoe_layer_cached_experts")
        return sorted(buf[i] for i in range(n.value))
