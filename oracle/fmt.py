"""ORACLE — test infrastructure only (tests/ and the fixture script).

Restatement of the reference's on-disk offload format:

* ``zipmoe_param`` (``csrc/tensor_engine/tensor_engine.cpp:139-220``): for a
  sparse (expert) tensor, each LZ4 exponent chunk is appended, then the raw
  sign+mantissa plane; every append is padded with zeros to a 4096-byte
  boundary (``OS_PAGE_SIZE``, ``tensor_engine.hpp:53``) and records the offset
  it started at.  Dense tensors append their raw bytes
  (``tensor_engine.cpp:303-316``) and store the offset in ``sm_file_offset``.
* ``zipmoe_index`` (``csrc/base/zipmoe_tensor_index.cpp:22-184``): native
  endian; ``u32 count`` then per entry ``u32 key`` followed by the
  ``TensorStorageMeta`` stream: ``u32 id; i64 ndim; i64 dims[ndim]; u64 size;
  u64 num_elements; u8 pinned; u8 requires_grad; i8 dtype; i8 device_index;
  i8 device_type; i8 layout; u32 offload_file_id; i32 num_file_chunks;
  (u32 k; u64 exp_file_offsets[k]); (u32 k; u64 compressed_sizes[k]);
  (u32 k; u64 original_sizes[k]); u64 sm_file_offset; u64 sm_size``.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Dict, List

PAGE = 4096
BF16_SCALAR_TYPE = 15   # c10::ScalarType::BFloat16


@dataclass
class Meta:
    id: int
    shape: List[int]
    size: int
    num_elements: int
    pinned: int = 0
    requires_grad: int = 0
    dtype: int = BF16_SCALAR_TYPE
    device_index: int = -1
    device_type: int = 0
    layout: int = 0
    offload_file_id: int = 0
    num_file_chunks: int = 0
    exp_file_offsets: List[int] = field(default_factory=list)
    compressed_sizes: List[int] = field(default_factory=list)
    original_sizes: List[int] = field(default_factory=list)
    sm_file_offset: int = 0
    sm_size: int = 0


def pack_meta(m: Meta) -> bytes:
    b = struct.pack("<I", m.id)
    b += struct.pack("<q", len(m.shape)) + b"".join(struct.pack("<q", d) for d in m.shape)
    b += struct.pack("<QQ", m.size, m.num_elements)
    b += struct.pack("<BBbbbb", m.pinned, m.requires_grad, m.dtype, m.device_index, m.device_type, m.layout)
    b += struct.pack("<Ii", m.offload_file_id, m.num_file_chunks)
    for arr in (m.exp_file_offsets, m.compressed_sizes, m.original_sizes):
        b += struct.pack("<I", len(arr)) + b"".join(struct.pack("<Q", v) for v in arr)
    b += struct.pack("<QQ", m.sm_file_offset, m.sm_size)
    return b


def serialize_index(entries: Dict[int, Meta]) -> bytes:
    out = struct.pack("<I", len(entries))
    for key, m in entries.items():
        out += struct.pack("<I", key) + pack_meta(m)
    return out


def deserialize_index(data: bytes) -> Dict[int, Meta]:
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from(fmt, data, pos)
        pos += struct.calcsize(fmt)
        return v

    (count,) = take("<I")
    out = {}
    for _ in range(count):
        (key,) = take("<I")
        (tid,) = take("<I")
        (ndim,) = take("<q")
        shape = list(take("<" + "q" * ndim)) if ndim else []
        size, nel = take("<QQ")
        pinned, rg, dt, di, dty, lay = take("<BBbbbb")
        fid, nfc = take("<Ii")
        arrs = []
        for _ in range(3):
            (k,) = take("<I")
            arrs.append(list(take("<" + "Q" * k)) if k else [])
        smo, sms = take("<QQ")
        out[key] = Meta(tid, shape, size, nel, pinned, rg, dt, di, dty, lay, fid, nfc,
                        arrs[0], arrs[1], arrs[2], smo, sms)
    return out


class ParamWriter:
    """Appends to an in-memory zipmoe_param image with the reference's padding."""

    def __init__(self):
        self.buf = bytearray()

    def append(self, data: bytes) -> int:
        start = len(self.buf)
        self.buf += data
        pad = (-len(self.buf)) % PAGE
        self.buf += b"\0" * pad
        return start

    def offload_sparse(self, tid: int, shape, blocks, original_sizes, sm: bytes) -> Meta:
        nel = 1
        for d in shape:
            nel *= d
        m = Meta(tid, list(shape), nel * 2, nel, num_file_chunks=len(blocks))
        m.original_sizes = list(original_sizes)
        m.compressed_sizes = [len(b) for b in blocks]
        m.exp_file_offsets = [self.append(b) for b in blocks]
        m.sm_size = len(sm)
        m.sm_file_offset = self.append(sm)
        return m

    def offload_dense(self, tid: int, shape, raw: bytes, num_file_chunks: int) -> Meta:
        nel = 1
        for d in shape:
            nel *= d
        m = Meta(tid, list(shape), len(raw), nel, num_file_chunks=num_file_chunks)
        m.exp_file_offsets = [0] * num_file_chunks
        m.compressed_sizes = [0] * num_file_chunks
        m.original_sizes = [0] * num_file_chunks
        m.sm_file_offset = self.append(raw)
        return m
