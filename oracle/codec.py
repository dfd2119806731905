"""ORACLE — test infrastructure only.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline /
reference leg may import this module, and only as the checker or as the timed
CPU baseline.  The product never imports it.

CPU restatement of the reference's expert codec:

* ``split_planes`` / ``chunk_exponents`` follow
  ``runtime/model_offload.py:706-726`` (``split_and_extract_from_tensor``):
  exponent plane ``(u16 >> 7) & 0xFF``, sign+mantissa plane
  ``((u16 >> 15) & 1) << 7 | (u16 & 0x7F)``, the exponent plane cut into
  ``num_file_chunks`` pieces of ``ceil(n / c)`` bytes (the last one shorter).
* ``lz4_compress_hc`` / ``lz4_compress_fast`` call liblz4 exactly as
  ``csrc/tensor_engine/compressors.cpp:105-122`` (``LZ4_compress_HC``, level 9
  in the evaluated configs) and ``:167-185`` (``LZ4_compress_fast``) do.
* ``lz4_decompress`` calls ``LZ4_decompress_safe_partial(src, dst, csize,
  osize, osize)`` as ``compressors.cpp:195-211`` does; ``lz4_decompress_restated``
  runs the C restatement in ``oracle/lz4_block.c`` on the same block.
* ``recombine`` follows ``csrc/kernels/tensor_recover.cu:25-30``.
* ``lz4_encode_chains`` is a serial statement of the GPU LZ4 encoder (a
  different encoder from liblz4's LZ4HC, whose blocks any LZ4 decoder reads);
  it is pinned by liblz4's decoder restoring every block it writes.

liblz4 is the reference's third-party codec (``csrc/CMakeLists.txt:37``; the
reference pins no version).  The image ships liblz4 1.9.4 as a runtime
library only, which is what these ctypes bindings load.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))

_lz4 = None
_orc = None


def liblz4() -> ctypes.CDLL:
    global _lz4
    if _lz4 is None:
        lib = ctypes.CDLL("liblz4.so.1")
        lib.LZ4_versionString.restype = ctypes.c_char_p
        lib.LZ4_compressBound.restype = ctypes.c_int
        lib.LZ4_compressBound.argtypes = [ctypes.c_int]
        for name in ("LZ4_compress_HC", "LZ4_compress_fast"):
            f = getattr(lib, name)
            f.restype = ctypes.c_int
            f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.LZ4_decompress_safe_partial.restype = ctypes.c_int
        lib.LZ4_decompress_safe_partial.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _lz4 = lib
    return _lz4


def lz4_version() -> str:
    return liblz4().LZ4_versionString().decode()


def _oracle_lib() -> ctypes.CDLL:
    global _orc
    if _orc is None:
        path = os.path.join(_HERE, "_build", "liboracle.so")
        if not os.path.exists(path):
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
        lib = ctypes.CDLL(path)
        lib.zmoe_oracle_lz4_decode.restype = ctypes.c_int
        lib.zmoe_oracle_lz4_decode.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
        lib.zmoe_oracle_lz4_encode_chains.restype = ctypes.c_int
        lib.zmoe_oracle_lz4_encode_chains.argtypes = [
            ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int]
        lib.zmoe_oracle_recombine.restype = None
        lib.zmoe_oracle_recombine.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        _orc = lib
    return _orc


# --------------------------------------------------------------------------
# planes
# --------------------------------------------------------------------------
def bf16_bits(x) -> np.ndarray:
    """uint16 bit patterns of a bf16 torch tensor (or a uint16 array)."""
    if isinstance(x, np.ndarray):
        return x.astype(np.uint16, copy=False).ravel()
    import torch
    return x.detach().contiguous().view(torch.int16).numpy().view(np.uint16).ravel()


def split_planes(bits: np.ndarray) -> Tuple[np.ndarray, np.ndarray]:
    """runtime/model_offload.py:711-714."""
    u = bits.astype(np.uint16, copy=False).ravel()
    exp = ((u >> 7) & 0xFF).astype(np.uint8)
    sm = ((((u >> 15) & 0x1) << 7) | (u & 0x7F)).astype(np.uint8)
    return np.ascontiguousarray(exp), np.ascontiguousarray(sm)


def chunk_exponents(exp: np.ndarray, num_file_chunks: int) -> List[np.ndarray]:
    """runtime/model_offload.py:717-724: ceil(n/c) bytes per chunk, last shorter."""
    n = exp.size
    per = (n + num_file_chunks - 1) // num_file_chunks
    out = []
    for c in range(num_file_chunks):
        s = c * per
        e = min(n, (c + 1) * per)
        out.append(exp[s:e].copy())
    return out


def recombine(exp: np.ndarray, sm: np.ndarray) -> np.ndarray:
    """csrc/kernels/tensor_recover.cu:25-30 (numpy form)."""
    s = sm.astype(np.uint16)
    return (((s >> 7) << 15) | (exp.astype(np.uint16) << 7) | (s & 0x7F)).astype(np.uint16)


def recombine_restated(exp: np.ndarray, sm: np.ndarray) -> np.ndarray:
    """Same as ``recombine`` through the C restatement."""
    exp = np.ascontiguousarray(exp, dtype=np.uint8)
    sm = np.ascontiguousarray(sm, dtype=np.uint8)
    out = np.empty(exp.size, dtype=np.uint16)
    _oracle_lib().zmoe_oracle_recombine(exp.ctypes.data, sm.ctypes.data, out.ctypes.data, exp.size)
    return out


# --------------------------------------------------------------------------
# LZ4 block codec
# --------------------------------------------------------------------------
def lz4_compress_hc(chunk: np.ndarray, level: int = 9) -> bytes:
    """compressors.cpp:105-122 (LZ4_compress_HC into a LZ4_compressBound buffer)."""
    lib = liblz4()
    src = np.ascontiguousarray(chunk, dtype=np.uint8)
    bound = lib.LZ4_compressBound(src.size)
    dst = ctypes.create_string_buffer(max(bound, 1))
    n = lib.LZ4_compress_HC(src.ctypes.data, ctypes.addressof(dst), src.size, bound, level)
    if n <= 0:
        raise RuntimeError("[LZ4HC] Compression Failed!")
    return dst.raw[:n]


def lz4_compress_fast(chunk: np.ndarray, acceleration: int = 5) -> bytes:
    """compressors.cpp:167-185 (LZ4_compress_fast)."""
    lib = liblz4()
    src = np.ascontiguousarray(chunk, dtype=np.uint8)
    bound = lib.LZ4_compressBound(src.size)
    dst = ctypes.create_string_buffer(max(bound, 1))
    n = lib.LZ4_compress_fast(src.ctypes.data, ctypes.addressof(dst), src.size, bound, acceleration)
    if n <= 0:
        raise RuntimeError("[LZ4] Compression Failed!")
    return dst.raw[:n]


def lz4_encode_chains(chunk: np.ndarray, attempts: int = 256) -> bytes:
    """Serial statement of the GPU encoder's parse (``lz4_block.c``), the
    bit-exact check of ``zmoe_lz4_encode_chains``'s blocks."""
    src = np.ascontiguousarray(chunk, dtype=np.uint8)
    cap = src.size + src.size // 255 + 16
    dst = np.zeros(max(cap, 1), dtype=np.uint8)
    n = _oracle_lib().zmoe_oracle_lz4_encode_chains(src.ctypes.data, src.size, dst.ctypes.data, cap, attempts)
    if n <= 0:
        raise RuntimeError("oracle lz4 encode failed")
    return dst[:n].tobytes()


def lz4_decompress(block: bytes, original_size: int) -> np.ndarray:
    """compressors.cpp:195-211: LZ4_decompress_safe_partial(src,dst,csize,osize,osize)."""
    lib = liblz4()
    out = np.zeros(original_size, dtype=np.uint8)
    src = ctypes.create_string_buffer(bytes(block), len(block))
    n = lib.LZ4_decompress_safe_partial(ctypes.addressof(src), out.ctypes.data, len(block),
                                        original_size, original_size)
    if n <= 0 and original_size > 0:
        raise RuntimeError("[LZ4] Decompression failed!")
    return out


def lz4_decompress_restated(block: bytes, original_size: int) -> Tuple[int, np.ndarray]:
    """oracle/lz4_block.c on the same block; returns (status_or_size, bytes)."""
    out = np.zeros(max(original_size, 1), dtype=np.uint8)
    src = ctypes.create_string_buffer(bytes(block), max(len(block), 1))
    n = _oracle_lib().zmoe_oracle_lz4_decode(ctypes.addressof(src), len(block), out.ctypes.data,
                                             original_size, original_size)
    return n, out[:original_size]


def lz4_sequences(block: bytes):
    """Token walk of one LZ4 block: list of (in_pos, out_pos, lit_len, offset, match_len).

    Used by tests for statistics and to pick adversarial cases; offset and
    match_len are 0 for the final literals-only sequence.
    """
    b = block
    n = len(b)
    i = 0
    op = 0
    seqs = []
    while i < n:
        start = i
        tok = b[i]
        i += 1
        ll = tok >> 4
        if ll == 15:
            while True:
                x = b[i]
                i += 1
                ll += x
                if x != 255:
                    break
        i += ll
        if i >= n:
            seqs.append((start, op, ll, 0, 0))
            op += ll
            break
        off = b[i] | (b[i + 1] << 8)
        i += 2
        ml = tok & 15
        if ml == 15:
            while True:
                x = b[i]
                i += 1
                ml += x
                if x != 255:
                    break
        ml += 4
        seqs.append((start, op, ll, off, ml))
        op += ll + ml
    return seqs


# --------------------------------------------------------------------------
# whole-tensor helpers
# --------------------------------------------------------------------------
def encode_tensor(bits: np.ndarray, num_file_chunks: int = 3, codec: str = "LZ4HC",
                  level: int = 9, acceleration: int = 5):
    """Split + chunk + compress one BF16 tensor; returns (blocks, original_sizes, sm)."""
    exp, sm = split_planes(bits)
    chunks = chunk_exponents(exp, num_file_chunks)
    blocks = []
    for c in chunks:
        if codec == "LZ4HC":
            blocks.append(lz4_compress_hc(c, level))
        elif codec == "LZ4":
            blocks.append(lz4_compress_fast(c, acceleration))
        else:
            raise ValueError(f"unsupported codec {codec}")
    return blocks, [c.size for c in chunks], sm


class Encoded:
    """One tensor in the reference's storage form (blocks, original sizes, sm bytes)."""

    def __init__(self, shape, blocks, original_sizes, sm: bytes):
        self.shape = tuple(shape)
        self.blocks = blocks
        self.original_sizes = list(original_sizes)
        self.sm = sm

    @property
    def numel(self) -> int:
        return sum(self.original_sizes)


def encode_tensors(tensors, num_file_chunks: int = 3, codec: str = "LZ4HC", level: int = 9,
                   threads: int = 0) -> List[Encoded]:
    """encode_tensor over many BF16 tensors, one chunk per task on a thread pool
    (the reference compresses on its compute pool, tensor_engine.cpp:223-301);
    ctypes releases the GIL inside each liblz4 call."""
    from concurrent.futures import ThreadPoolExecutor
    planes = []
    for t in tensors:
        exp, sm = split_planes(bf16_bits(t))
        planes.append((tuple(t.shape), chunk_exponents(exp, num_file_chunks), sm))
    jobs = [c for _, chunks, _ in planes for c in chunks]

    def one(c):
        if codec == "LZ4HC":
            return lz4_compress_hc(c, level)
        if codec == "LZ4":
            return lz4_compress_fast(c, level)
        raise ValueError(f"unsupported codec {codec}")

    with ThreadPoolExecutor(max_workers=threads or (os.cpu_count() or 1)) as ex:
        blocks = list(ex.map(one, jobs))
    out, pos = [], 0
    for shape, chunks, sm in planes:
        out.append(Encoded(shape, blocks[pos:pos + len(chunks)], [c.size for c in chunks], sm.tobytes()))
        pos += len(chunks)
    return out


def decode_tensor(blocks: Sequence[bytes], original_sizes: Sequence[int], sm: np.ndarray) -> np.ndarray:
    """Reference CPU miss path: decode every chunk, concatenate, recombine."""
    exp = np.concatenate([lz4_decompress(b, o) for b, o in zip(blocks, original_sizes)])
    return recombine(exp, sm)
