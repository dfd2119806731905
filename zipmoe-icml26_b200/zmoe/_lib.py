"""ctypes binding of libzmoe.so (the C ABI declared in include/zmoe.h).

The library is built in place by ``make`` in the package directory.  There is
no fallback: if the library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libzmoe.so")

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_u32 = ctypes.c_uint32
c_size_t = ctypes.c_size_t
c_float = ctypes.c_float


class ZmoeChunk(ctypes.Structure):
    _fields_ = [("src", c_void_p), ("sm", c_void_p), ("dst", c_void_p), ("index", c_void_p), ("map", c_void_p),
                ("src_size", c_u32), ("out_size", c_u32), ("n_index", c_u32), ("seg_bytes", c_u32)]


class ZmoeEncChunk(ctypes.Structure):
    _fields_ = [("src", c_void_p), ("dst", c_void_p), ("scratch", c_void_p),
                ("src_size", c_u32), ("dst_capacity", c_u32)]


SLICE_BYTES = 256        # ZMOE_SLICE_BYTES
MAP_ENTRIES = 65536      # ZMOE_MAP_ENTRIES (per 64 KiB region)


class RouterArgs(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("w", c_void_p), ("bias", c_void_p), ("w_shared_gate", c_void_p),
                ("T", c_int), ("H", c_int), ("E", c_int), ("k", c_int), ("mode", c_int),
                ("norm_topk_prob", c_int), ("scaling", c_float),
                ("logits", c_void_p), ("topk_idx", c_void_p), ("topk_w", c_void_p), ("shared_gate", c_void_p)]


class PermuteArgs(ctypes.Structure):
    _fields_ = [("topk_idx", c_void_p), ("x", c_void_p), ("T", c_int), ("H", c_int), ("E", c_int),
                ("k", c_int), ("capacity", c_int), ("seq_len", c_int), ("counts", c_void_p),
                ("offsets", c_void_p), ("row_of", c_void_p), ("token_of_row", c_void_p), ("xp", c_void_p)]


class FfnArgs(ctypes.Structure):
    _fields_ = [("x", c_void_p), ("w", c_void_p), ("offsets", c_void_p), ("G", c_int),
                ("rows_total", c_int), ("H", c_int), ("I", c_int), ("kind", c_int),
                ("h", c_void_p), ("y", c_void_p)]


class CombineArgs(ctypes.Structure):
    _fields_ = [("y", c_void_p), ("y_shared", c_void_p), ("shared_gate", c_void_p), ("row_of", c_void_p),
                ("topk_w", c_void_p), ("x", c_void_p), ("T", c_int), ("H", c_int), ("k", c_int),
                ("mode", c_int), ("out", c_void_p)]


class LayerConfig(ctypes.Structure):
    _fields_ = [("hidden", c_int), ("num_experts", c_int), ("inter", c_int), ("topk", c_int),
                ("kind", c_int), ("route_mode", c_int), ("norm_topk_prob", c_int), ("scaling", c_float),
                ("shared_inter", c_int), ("capacity", c_int), ("seq_len", c_int), ("max_tokens", c_int),
                ("cache_slots", c_int), ("transient_slots", c_int), ("cache_policy", c_int),
                ("state_margin", ctypes.c_double), ("sm_slots", c_int)]


class LayerStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in (
        "forwards", "tokens", "hits", "misses", "evictions", "decoded_experts", "decoded_chunks",
        "decoded_bytes", "decode_launches", "launches", "decode_errors", "store_bytes",
        "decode_ns", "decode_timed_bytes", "decode_timed_launches", "ffn_ns", "ffn_timed_launches",
        "host_copy_bytes", "sm_resident_tensors")]


class EPConfig(ctypes.Structure):
    _fields_ = [("layer", LayerConfig), ("rank", c_int), ("world", c_int), ("nccl_comm", c_void_p)]


# (name, restype, argtypes) of every exported symbol; tests check the header
# declares exactly these.
SIGNATURES = {
    "zmoe_abi_version": (c_int, []),
    "zmoe_last_error": (ctypes.c_char_p, []),
    "zmoe_kernel_error": (c_int, [ctypes.POINTER(ctypes.c_int32), c_int]),
    "zmoe_debug_ffn_wait": (c_int, [ctypes.c_longlong, c_int]),
    "zmoe_clock_probe": (c_int, [c_void_p, ctypes.c_uint64, c_void_p]),
    "zmoe_tensor_recover": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "zmoe_decode_chunks": (c_int, [c_void_p, c_int, c_void_p, c_void_p]),
    "zmoe_decode_scratch_bytes": (ctypes.c_uint64, [c_u32]),
    "zmoe_router": (c_int, [ctypes.POINTER(RouterArgs), c_void_p]),
    "zmoe_permute": (c_int, [ctypes.POINTER(PermuteArgs), c_void_p]),
    "zmoe_expert_ffn": (c_int, [ctypes.POINTER(FfnArgs), c_void_p]),
    "zmoe_expert_ffn_noalloc": (c_int, [ctypes.POINTER(FfnArgs), c_void_p]),
    "zmoe_combine": (c_int, [ctypes.POINTER(CombineArgs), c_void_p]),
    "zmoe_gather_rows": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "zmoe_split_planes": (c_int, [c_void_p, ctypes.c_uint64, c_void_p, c_void_p]),
    "zmoe_lz4_compress_bound": (c_int, [c_int]),
    "zmoe_lz4_compress": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int]),
    "zmoe_lz4_build_index": (c_int, [c_void_p, c_u32, c_u32, c_u32, c_void_p, c_int]),
    "zmoe_lz4_encode_chunks": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    "zmoe_lz4_encode_scratch_bytes": (ctypes.c_uint64, [c_u32]),
    "zmoe_layer_create": (c_int, [ctypes.POINTER(LayerConfig), ctypes.POINTER(c_void_p)]),
    "zmoe_layer_destroy": (c_int, [c_void_p]),
    "zmoe_layer_set_router": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "zmoe_layer_set_shared": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "zmoe_layer_load_expert": (c_int, [c_void_p, c_int, c_int, ctypes.POINTER(c_void_p),
                                       ctypes.POINTER(c_u32), ctypes.POINTER(c_u32), c_int, c_void_p,
                                       ctypes.c_uint64]),
    "zmoe_layer_warm_cache": (c_int, [c_void_p, ctypes.POINTER(c_int), c_int, c_void_p]),
    "zmoe_layer_set_store": (c_int, [c_void_p, c_int]),
    "zmoe_layer_forward": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "zmoe_layer_experts": (c_int, [c_void_p, c_void_p, ctypes.POINTER(ctypes.c_int32), c_int, c_void_p, c_void_p]),
    "zmoe_layer_forward_host": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "zmoe_layer_submit_host": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    "zmoe_layer_join_host": (c_int, [c_void_p, c_void_p]),
    "zmoe_layer_sync": (c_int, [c_void_p, c_void_p]),
    "zmoe_layer_get_stats": (c_int, [c_void_p, ctypes.POINTER(LayerStats)]),
    "zmoe_layer_reset_stats": (c_int, [c_void_p]),
    "zmoe_layer_set_timing": (c_int, [c_void_p, c_int]),
    "zmoe_layer_reset_access_counts": (c_int, [c_void_p]),
    "zmoe_layer_prefetch": (c_int, [c_void_p, ctypes.POINTER(c_int), c_int, c_void_p]),
    "zmoe_layer_last_counts": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_int32), c_int, ctypes.POINTER(c_int)]),
    "zmoe_layer_cached_experts": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_int32), c_int,
                                          ctypes.POINTER(c_int)]),
    "zmoe_ep_create": (c_int, [ctypes.POINTER(EPConfig), c_void_p, ctypes.POINTER(c_void_p)]),
    "zmoe_ep_destroy": (c_int, [c_void_p]),
    "zmoe_ep_set_router": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "zmoe_ep_set_shared": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "zmoe_ep_forward": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
}


class ZmoeError(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libzmoe.so not built ({LIB_PATH}); run `make` in {PKG_DIR}")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    return lib


lib = _load()


def check(status: int, what: str):
    if status != 0:
        raise ZmoeError(f"{what}: status {status}: {lib.zmoe_last_error().decode(errors='replace')}")
