"""Offload-side encoding of expert tensors into the reference's storage form.

Split into planes (runtime/model_offload.py:706-726), cut the exponent plane
into ``num_file_chunks`` chunks of ceil(n/c) bytes, LZ4-compress each chunk
(csrc/tensor_engine/compressors.cpp:105-122 / :167-185) — all through
libzmoe.so.  Encoding many tensors runs chunks on a thread pool, as the
reference's compute pool does (tensor_engine.cpp:223-301); ctypes releases the
GIL during each call.
"""
from __future__ import annotations

import ctypes
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np
import torch

from ._lib import lib

CODECS = {"LZ4": 0, "LZ4HC": 1}


@dataclass
class EncodedTensor:
    """One tensor in the reference's storage form."""
    shape: tuple
    blocks: List[bytes]
    original_sizes: List[int]
    sm: bytes

    @property
    def numel(self) -> int:
        return sum(self.original_sizes)

    @property
    def compressed_bytes(self) -> int:
        return sum(len(b) for b in self.blocks)


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).ravel()


def split_planes(bits: np.ndarray):
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    exp = np.empty(bits.size, np.uint8)
    sm = np.empty(bits.size, np.uint8)
    rc = lib.zmoe_split_planes(bits.ctypes.data, bits.size, exp.ctypes.data, sm.ctypes.data)
    if rc:
        raise RuntimeError("zmoe_split_planes failed")
    return exp, sm


def compress_chunk(chunk: np.ndarray, codec: str = "LZ4HC", level: int = 9) -> bytes:
    chunk = np.ascontiguousarray(chunk, dtype=np.uint8)
    cap = lib.zmoe_lz4_compress_bound(chunk.size)
    if cap <= 0:
        raise RuntimeError("liblz4 is not available")
    dst = ctypes.create_string_buffer(max(cap, 1))
    n = lib.zmoe_lz4_compress(chunk.ctypes.data, chunk.size, ctypes.addressof(dst), cap, CODECS[codec], level)
    if n <= 0:
        raise RuntimeError(f"[{codec}] Compression Failed!")
    return dst.raw[:n]


def chunk_bounds(n: int, num_file_chunks: int):
    per = (n + num_file_chunks - 1) // num_file_chunks
    return [(c * per, min(n, (c + 1) * per)) for c in range(num_file_chunks)]


def encode_tensors(tensors: Sequence[torch.Tensor], num_file_chunks: int = 3, codec: str = "LZ4HC",
                   level: int = 9, threads: int = 0) -> List[EncodedTensor]:
    """Encode BF16 tensors; LZ4HC level = compression level, LZ4 level = acceleration."""
    planes = []
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise ValueError("expert tensors must be BF16")
        exp, sm = split_planes(bf16_bits(t))
        planes.append((tuple(t.shape), exp, sm))
    jobs = []
    for ti, (_, exp, _) in enumerate(planes):
        for c, (a, b) in enumerate(chunk_bounds(exp.size, num_file_chunks)):
            jobs.append((ti, c, exp[a:b]))
    threads = threads or min(32, os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=threads) as ex:
        blocks = list(ex.map(lambda j: compress_chunk(j[2], codec, level), jobs))
    out = []
    pos = 0
    for shape, exp, sm in planes:
        bounds = chunk_bounds(exp.size, num_file_chunks)
        out.append(EncodedTensor(shape, blocks[pos:pos + len(bounds)], [b - a for a, b in bounds], sm.tobytes()))
        pos += len(bounds)
    return out
