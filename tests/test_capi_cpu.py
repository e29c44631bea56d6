"""The C ABI library loads without a GPU and exports every entry point include/lbq.h declares."""
import ctypes
import os
import re

from lingbot_b200 import _lib
from lingbot_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    src = open(os.path.join(ROOT, "include", "lbq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(lbq_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_expected_entry_points():
    names = declared()
    for n in ("lbq_quant_qkv", "lbq_requant_cache", "lbq_attn_fwd", "lbq_splitkv_combine", "lbq_last_error"):
        assert n in names


def test_library_loads_and_exports_every_declared_symbol():
    build()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_ctypes_signatures_cover_the_header():
    assert sorted(_lib.SIGNATURES) == declared()


def test_argument_validation_without_a_gpu():
    """Host-side checks fire before any CUDA call: errors come back as codes + messages."""
    _lib.load()
    lib = _lib._lib
    rc = lib.lbq_quant_q(None, 0, 0, 0, 1, 1, 1, None, None, None)
    assert rc == 1 and b"null" in lib.lbq_last_error()
    buf = ctypes.create_string_buffer(64)
    mis = ctypes.c_void_p(ctypes.addressof(buf) + 1)
    rc = lib.lbq_quant_q(mis, 0, 0, 0, 1, 1, 1, mis, mis, None)
    assert rc == 2 and b"aligned" in lib.lbq_last_error()
    assert lib.lbq_abi_version() == 101


def test_quant_workspace_size_is_checked():
    """lbq_quant_qkv_workspace: the documented size, and SIZE_MAX (so every capacity check rejects the
    call) for out-of-range arguments or a size that would overflow."""
    lib = _lib.load()
    ws = lib.lbq_quant_qkv_workspace
    size_max = ctypes.c_size_t(-1).value
    assert ws(1, 12, 30160) == 1 * 12 * ((30160 + 63) // 64 + 1) * 1536 + 64
    assert ws(1, 12, 58176) <= 16 << 20 < ws(1, 12, 58176 + 64)
    for args in [(0, 12, 100), (1, 0, 100), (70000, 1, 100), (1, 70000, 100), (1, 12, 0), (1, 12, (1 << 30) + 1),
                 (65535, 65535, 1 << 30)]:
        assert ws(*args) == size_max, args



def test_debug_library_exports_the_same_entry_points():
    """liblbq_debug.so (device-side index checks, LBQ_DEBUG_LIB=1) exports every declared entry point."""
    from lingbot_b200 import build as b
    path = b.build(debug=True)
    lib = ctypes.CDLL(path)
    for name in declared():
        assert hasattr(lib, name), name
    assert lib.lbq_abi_version() == _lib.load().lbq_abi_version()
