"""The C ABI library loads and exports every symbol include/zmoe.h declares
(no GPU needed: nothing is launched)."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "zmoe.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(zmoe_\w+)\s*\(", src, flags=re.M))


def test_library_exports_header_symbols():
    from zmoe import _lib
    syms = header_symbols()
    assert "zmoe_decode_chunks" in syms and "zmoe_tensor_recover" in syms
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert set(_lib.SIGNATURES) <= syms | {"zmoe_last_error", "zmoe_abi_version"}
    assert lib.zmoe_abi_version() == 3


def test_struct_layouts_match_header():
    from zmoe import _lib
    assert ctypes.sizeof(_lib.ZmoeChunk) == 56
    # 4 pointers, 6 ints, 1 float (+4 padding), 4 pointers
    assert ctypes.sizeof(_lib.RouterArgs) == 96
    src = '#include "zmoe.h"\n#include <stdio.h>\nint main(){printf("%zu %zu %zu %zu %zu", sizeof(zmoe_chunk), sizeof(zmoe_router_args), sizeof(zmoe_permute_args), sizeof(zmoe_ffn_args), sizeof(zmoe_combine_args));}'
    import subprocess, tempfile
    with tempfile.TemporaryDirectory() as d:
        open(os.path.join(d, "s.c"), "w").write(src)
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), "-o", os.path.join(d, "s"), os.path.join(d, "s.c")], check=True)
        got = [int(v) for v in subprocess.run([os.path.join(d, "s")], capture_output=True, text=True, check=True).stdout.split()]
    assert got == [ctypes.sizeof(c) for c in (_lib.ZmoeChunk, _lib.RouterArgs, _lib.PermuteArgs, _lib.FfnArgs, _lib.CombineArgs)]


def test_argument_errors_need_no_gpu():
    from zmoe import _lib
    rc = _lib.lib.zmoe_decode_chunks(None, 3, None, None)
    assert rc == 1
    assert b"null" in _lib.lib.zmoe_last_error()
