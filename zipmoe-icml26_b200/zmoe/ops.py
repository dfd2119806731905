"""Torch-facing wrappers over the C ABI (device tensors in, device tensors out).

Every call runs on torch's current CUDA stream and raises ``ZmoeError`` with
the library's message on a non-zero status.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import CombineArgs, FfnArgs, PermuteArgs, RouterArgs, ZmoeChunk, ZmoeEncChunk, check, lib

ROUTE_QWEN, ROUTE_DEEPSEEK, ROUTE_SWITCH = 0, 1, 2


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, dtype, name: str):
    if not t.is_cuda or t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor, got {t.dtype} on {t.device}")


# ---------------------------------------------------------------------------
# codec
# ---------------------------------------------------------------------------
def tensor_recover(exp: torch.Tensor, sm: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """BF16 bits from the exponent and sign+mantissa planes (uint8 -> int16 view)."""
    _need(exp, torch.uint8, "exp")
    _need(sm, torch.uint8, "sm")
    if exp.numel() != sm.numel():
        raise ValueError("plane sizes differ")
    if out is None:
        out = torch.empty(exp.numel(), dtype=torch.bfloat16, device=exp.device)
    check(lib.zmoe_tensor_recover(out.data_ptr(), exp.data_ptr(), sm.data_ptr(), exp.numel(), _stream()),
          "zmoe_tensor_recover")
    return out


SEG_BYTES = _lib.SLICE_BYTES


def scratch_bytes(out_size: int) -> int:
    """Decoder scratch of one indexed chunk (zmoe_decode_scratch_bytes)."""
    return int(lib.zmoe_decode_scratch_bytes(int(out_size)))


def map_scratch(out_sizes: Sequence[int], device) -> torch.Tensor:
    """Decoder scratch for indexed chunks of the given output sizes, in order."""
    total = sum(scratch_bytes(o) for o in out_sizes)
    return torch.empty(max(total, 16) // 4, dtype=torch.int32, device=device)


def chunk_table(descs: Sequence[tuple], device, scratch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Pack (src, sm, dst, src_size, out_size[, index, n_index, seg_bytes]) tuples
    into a device descriptor array; indexed chunks get consecutive scratch areas
    (map_scratch of the indexed chunks' out_sizes, in the same order)."""
    arr = (ZmoeChunk * max(len(descs), 1))()
    off = 0
    for i, d in enumerate(descs):
        src, sm, dst, csz, osz = d[:5]
        idx, nidx, seg = d[5:8] if len(d) >= 8 else (None, 0, 0)
        mp = None
        if idx and scratch is not None:
            mp = scratch.data_ptr() + off
            off += scratch_bytes(osz)
        arr[i] = ZmoeChunk(src, sm, dst, idx, mp, csz, osz, nidx, seg)
    size = ctypes.sizeof(ZmoeChunk)
    raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)[: size * len(descs)]
    return raw.to(device)


def build_index(block: bytes, out_size: int, seg_bytes: int = SEG_BYTES) -> np.ndarray:
    """Segment index of one LZ4 block (uint32 [n, 2])."""
    n = max(1, (out_size + seg_bytes - 1) // seg_bytes)
    ent = np.zeros((n, 2), np.uint32)
    buf = ctypes.create_string_buffer(bytes(block), max(len(block), 1))
    rc = lib.zmoe_lz4_build_index(ctypes.addressof(buf), len(block), out_size, seg_bytes, ent.ctypes.data, n)
    if rc < 0:
        raise ValueError(f"zmoe_lz4_build_index failed ({rc})")
    return ent[:rc]


def decode_chunks(table: torch.Tensor, n: int, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Launch the fused decoder on a device descriptor table; returns int32 status[n]."""
    if status is None:
        status = torch.full((max(n, 1),), -1, dtype=torch.int32, device=table.device)
    check(lib.zmoe_decode_chunks(table.data_ptr(), n, status.data_ptr(), _stream()), "zmoe_decode_chunks")
    return status[:n]


def lz4_encode_chunks(chunks: Sequence[torch.Tensor], max_attempts: int = 256) -> List[torch.Tensor]:
    """LZ4 blocks of uint8 device chunks, all encoded in one zmoe_lz4_encode_chunks
    launch (replaces LZ4HCcompressor::compress, csrc/tensor_engine/compressors.cpp:105-122,
    run per chunk on the CPU).  Returns one uint8 device tensor per chunk (views
    into one buffer); waits once for the block sizes."""
    if not chunks:
        return []
    dev = chunks[0].device
    for c in chunks:
        _need(c, torch.uint8, "chunk")
    caps = [c.numel() + c.numel() // 255 + 16 for c in chunks]
    scr = [(int(lib.zmoe_lz4_encode_scratch_bytes(c.numel())) + 15) // 16 * 16 for c in chunks]
    dst = torch.empty(sum(caps), dtype=torch.uint8, device=dev)
    scratch = torch.empty(max(sum(scr), 16) // 16, 2, dtype=torch.int64, device=dev)   # 16-byte aligned
    arr = (ZmoeEncChunk * len(chunks))()
    doff = soff = 0
    for i, c in enumerate(chunks):
        arr[i] = ZmoeEncChunk(c.data_ptr(), dst.data_ptr() + doff, scratch.data_ptr() + soff, c.numel(), caps[i])
        doff += caps[i]
        soff += scr[i]
    table = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8).to(dev)
    sizes = torch.zeros(len(chunks), dtype=torch.int32, device=dev)
    check(lib.zmoe_lz4_encode_chunks(table.data_ptr(), len(chunks), int(max_attempts), sizes.data_ptr(), _stream()),
          "zmoe_lz4_encode_chunks")
    host = sizes.cpu().tolist()
    out, doff = [], 0
    for i, n in enumerate(host):
        if n <= 0:
            raise _lib.ZmoeError(f"zmoe_lz4_encode_chunks: chunk {i} did not encode")
        out.append(dst[doff:doff + n])
        doff += caps[i]
    return out


def _split_exponents(bits: torch.Tensor, num_file_chunks: int):
    """Exponent plane cut into num_file_chunks pieces of ceil(n / c) bytes (the
    last shorter) and the sign+mantissa plane (runtime/model_offload.py:706-726)."""
    if not bits.is_cuda or bits.dtype not in (torch.bfloat16, torch.int16):
        raise ValueError("encode: expected a CUDA bfloat16 tensor")
    u = bits.contiguous().view(torch.int16).reshape(-1).to(torch.int32) & 0xFFFF
    exp = ((u >> 7) & 0xFF).to(torch.uint8)
    sm = (((u >> 15) & 1) << 7 | (u & 0x7F)).to(torch.uint8)
    n = exp.numel()
    per = -(-n // num_file_chunks)
    return [exp[min(n, c * per):min(n, (c + 1) * per)] for c in range(num_file_chunks)], sm


def encode_tensor(bits: torch.Tensor, num_file_chunks: int = 3, max_attempts: int = 256):
    """Offload form of one BF16 tensor on the GPU: the exponent plane cut into
    num_file_chunks LZ4 blocks and the sign+mantissa plane
    (runtime/model_offload.py:706-726, then TensorEngine::PipelineCompress).
    bits: BF16 (or its int16 view) on the device.  Returns (blocks as device
    tensors, original_sizes, sm as a device uint8 tensor)."""
    return encode_tensors([bits], num_file_chunks, max_attempts)[0]


def encode_tensors(tensors: Sequence[torch.Tensor], num_file_chunks: int = 3, max_attempts: int = 256):
    """encode_tensor for many tensors, every chunk of every tensor in one
    zmoe_lz4_encode_chunks launch (TensorEngine::PipelineCompress's chunks all
    at once).  Returns [(blocks, original_sizes, sm)] in order."""
    split = [_split_exponents(t, num_file_chunks) for t in tensors]
    blocks = lz4_encode_chunks([p for pieces, _ in split for p in pieces], max_attempts)
    out = []
    for k, (pieces, sm) in enumerate(split):
        out.append((blocks[k * num_file_chunks:(k + 1) * num_file_chunks], [p.numel() for p in pieces], sm))
    return out


class CompressedTensor:
    """One expert matrix in HBM in the reference's storage form: LZ4 exponent
    chunks (concatenated, 16-byte aligned) and the raw sign+mantissa plane."""

    def __init__(self, blocks: Sequence[bytes], original_sizes: Sequence[int], sm: bytes, device="cuda",
                 seg_bytes: int = SEG_BYTES, indexed: bool = True):
        self.original_sizes = [int(o) for o in original_sizes]
        self.compressed_sizes = [len(b) for b in blocks]
        self.numel = sum(self.original_sizes)
        self.seg_bytes = seg_bytes
        offs, pos = [], 0
        for b in blocks:
            offs.append(pos)
            pos += (len(b) + 15) // 16 * 16
        buf = bytearray(max(pos, 16))
        for o, b in zip(offs, blocks):
            buf[o:o + len(b)] = b
        self.block_offsets = offs
        self.blocks = torch.frombuffer(buf, dtype=torch.uint8).to(device)
        self.sm = torch.frombuffer(bytearray(sm), dtype=torch.uint8).to(device)
        self.indexes = None
        if indexed:
            idx = [build_index(b, o, seg_bytes) for b, o in zip(blocks, self.original_sizes)]
            self.index_rows = [len(i) for i in idx]
            flat = np.concatenate(idx) if idx else np.zeros((1, 2), np.uint32)
            self.indexes = torch.from_numpy(flat.astype(np.int32)).to(device)
            self.index_offsets = np.concatenate([[0], np.cumsum(self.index_rows)]).tolist()

    @property
    def device_bytes(self) -> int:
        return self.blocks.numel() + self.sm.numel() + (self.indexes.numel() * 4 if self.indexes is not None else 0)

    def descs(self, dst: torch.Tensor) -> List[tuple]:
        out, e0 = [], 0
        for i, (o, c, n) in enumerate(zip(self.block_offsets, self.compressed_sizes, self.original_sizes)):
            d = (self.blocks.data_ptr() + o, self.sm.data_ptr() + e0, dst.data_ptr() + 2 * e0, c, n)
            if self.indexes is not None:
                d = d + (self.indexes.data_ptr() + 8 * self.index_offsets[i], self.index_rows[i], self.seg_bytes)
            out.append(d)
            e0 += n
        return out

    def decode(self, dst: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        if dst is None:
            dst = torch.empty(self.numel, dtype=torch.bfloat16, device=self.blocks.device)
        d = self.descs(dst)
        scratch = map_scratch([x[4] for x in d], dst.device) if self.indexes is not None else None
        table = chunk_table(d, dst.device, scratch)
        st = decode_chunks(table, len(d))
        self._scratch = scratch                      # alive until the caller synchronises
        return dst, st


# ---------------------------------------------------------------------------
# layer primitives
# ---------------------------------------------------------------------------
def router(x: torch.Tensor, w: torch.Tensor, k: int, mode: int, bias: Optional[torch.Tensor] = None,
           w_shared_gate: Optional[torch.Tensor] = None, scaling: float = 1.0, norm_topk_prob: bool = False,
           want_logits: bool = True):
    _need(x, torch.bfloat16, "x")
    _need(w, torch.bfloat16, "w")
    T, H = x.shape
    E = w.shape[0]
    dev = x.device
    logits = torch.empty(T, E, dtype=torch.float32, device=dev) if want_logits else None
    idx = torch.empty(T, k, dtype=torch.int32, device=dev)
    tw = torch.empty(T, k, dtype=torch.float32, device=dev)
    sg = torch.empty(T, dtype=torch.float32, device=dev) if w_shared_gate is not None else None
    if bias is not None:
        _need(bias, torch.float32, "bias")
    a = RouterArgs(x.data_ptr(), w.data_ptr(), _ptr(bias), _ptr(w_shared_gate), T, H, E, k, mode,
                   int(norm_topk_prob), scaling, _ptr(logits), idx.data_ptr(), tw.data_ptr(), _ptr(sg))
    check(lib.zmoe_router(ctypes.byref(a), _stream()), "zmoe_router")
    return logits, idx, tw, sg


def permute(topk_idx: torch.Tensor, x: Optional[torch.Tensor], E: int, capacity: int = 0, seq_len: int = 0):
    """Returns counts, offsets, row_of, token_of_row, xp.  topk_idx is updated
    in place (-1 for capacity drops)."""
    _need(topk_idx, torch.int32, "topk_idx")
    T, k = topk_idx.shape
    dev = topk_idx.device
    H = x.shape[1] if x is not None else 0
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_of = torch.empty(T, k, dtype=torch.int32, device=dev)
    tor = torch.empty(max(T * k, 1), dtype=torch.int32, device=dev)
    xp = torch.empty(max(T * k, 1), H, dtype=torch.bfloat16, device=dev) if x is not None else None
    a = PermuteArgs(topk_idx.data_ptr(), _ptr(x), T, H, E, k, capacity, seq_len, counts.data_ptr(),
                    offsets.data_ptr(), row_of.data_ptr(), tor.data_ptr(), _ptr(xp))
    check(lib.zmoe_permute(ctypes.byref(a), _stream()), "zmoe_permute")
    return counts, offsets, row_of, tor, xp


def weight_table(mats: Sequence[Sequence[Optional[torch.Tensor]]], device=None) -> torch.Tensor:
    """Host array [G*3] of device weight pointers from per-group (w0, w1, w2)
    (the FFN builds one TMA descriptor per matrix on the host)."""
    ptrs = []
    for g in mats:
        g = list(g) + [None] * (3 - len(g))
        ptrs.extend(0 if t is None else t.data_ptr() for t in g)
    return torch.tensor(ptrs, dtype=torch.int64)


def expert_ffn(x: torch.Tensor, wtab: torch.Tensor, offsets: Optional[torch.Tensor], G: int, I: int, kind: int,
               rows_total: Optional[int] = None):
    _need(x, torch.bfloat16, "x")
    rows = x.shape[0] if rows_total is None else rows_total
    H = x.shape[1]
    h = torch.empty(max(rows, 1), I, dtype=torch.bfloat16, device=x.device)
    y = torch.empty(max(rows, 1), H, dtype=torch.bfloat16, device=x.device)
    a = FfnArgs(x.data_ptr(), wtab.data_ptr(), _ptr(offsets), G, rows, H, I, kind, h.data_ptr(), y.data_ptr())
    check(lib.zmoe_expert_ffn(ctypes.byref(a), _stream()), "zmoe_expert_ffn")
    return y, h


def combine(y: torch.Tensor, row_of: torch.Tensor, topk_w: torch.Tensor, mode: int,
            y_shared: Optional[torch.Tensor] = None, shared_gate: Optional[torch.Tensor] = None,
            x: Optional[torch.Tensor] = None, H: Optional[int] = None) -> torch.Tensor:
    T, k = row_of.shape
    H = y.shape[1] if H is None else H
    out = torch.empty(T, H, dtype=torch.bfloat16, device=y.device)
    a = CombineArgs(y.data_ptr(), _ptr(y_shared), _ptr(shared_gate), row_of.data_ptr(), topk_w.data_ptr(),
                    _ptr(x), T, H, k, mode, out.data_ptr())
    check(lib.zmoe_combine(ctypes.byref(a), _stream()), "zmoe_combine")
    return out
