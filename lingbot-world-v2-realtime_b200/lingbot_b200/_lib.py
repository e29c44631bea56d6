"""ctypes binding of liblbq.so (C ABI declared in include/lbq.h).

The library is loaded on first use; if it is missing or fails to load, every call raises — there is
no fallback implementation.
"""
import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.abspath(__file__))
# LBQ_DEBUG_LIB=1: the debug build (device-side index checks recording 0x3xx status codes)
LIB_PATH = os.path.join(_PKG, "liblbq_debug.so" if os.environ.get("LBQ_DEBUG_LIB") == "1" else "liblbq.so")

_i32, _i64, _f32, _vp, _sz = ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
_u64 = ctypes.c_uint64

# name -> (restype, argtypes)
SIGNATURES = {
    "lbq_abi_version": (_i32, []),
    "lbq_last_error": (ctypes.c_char_p, []),
    "lbq_device_status": (_i32, [_i32, ctypes.POINTER(_i32)]),
    "lbq_kv_block_stats": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i64, _i32, _i32,
                                  _i64, _vp, _vp, _i64, _i64, _i64, _vp]),
    "lbq_kv_window_sums": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _i64, _vp, _vp, _vp]),
    "lbq_quant_q": (_i32, [_vp, _i64, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "lbq_rope_quant_q": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _vp, _vp, _vp]),
    "lbq_cache_write": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _i64,
                               _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i64, _i64, _i64, _i64,
                               _vp, _vp, _i64, _i64, _i64, _vp]),
    "lbq_quant_kv": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i64, _i32, _i32, _i32, _i32,
                            _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp]),
    "lbq_quant_qkv_workspace": (_sz, [_i32, _i32, _i64]),
    "lbq_quant_qkv": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
                             _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i32, _vp]),
    "lbq_quant_qkv_static": (_i32, [_vp, _i64, _i64, _i64, _i32, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
                                    _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp]),
    "lbq_requant_cache": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i64, _i64, _vp, _vp,
                                 _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "lbq_attn_fwd": (_i32, [_vp, _vp, _i32, _vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _i64,
                            _i64, _i64, _i32, _vp, _vp, ctypes.POINTER(_i32), _i32, _vp]),
    "lbq_fp8_quant_rows": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _vp]),
    "lbq_fp8_gemm": (_i32, [_vp, _i64, _vp, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _vp, _i64, _i32, _vp]),
    "lbq_splitkv_combine": (_i32, [_vp, _vp, _i32, _vp, _i32, _i32, _i32, _vp, _i64, _i64, _i64, _i32, _vp]),
    "lbq_peer_export": (_i32, [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)]),
    "lbq_peer_open": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "lbq_peer_close": (_i32, [_vp]),
    "lbq_exchange_bytes": (_i64, [_i32, _i32, _i32]),
    "lbq_share_totals_push": (_i32, [_vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _i64, _vp]),
    "lbq_chunk_totals": (_i32, [_vp, _i32, _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _u64, _vp]),
    "lbq_share_push": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _i32,
                              _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _vp]),
    "lbq_share_quant_push": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i32, _i32, _i32,
                                    _i32, _i32, _i32, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _i32,
                                    _i32, _i64, _i32, _vp]),
    "lbq_peer_wait": (_i32, [_vp, _i32, _i32, _i64, _i32, _u64, _vp]),
    "lbq_quant_kv_tiles": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i64, _i32, _i32, _i32,
                                  _i32, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "lbq_attn_fwd_keys": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _vp, _vp,
                                 _vp, _i32, _i32, _i64, _i32, _i64, _i64, _vp]),
    "lbq_keys_combine": (_i32, [_vp, _vp, _i32, _i32, _i32, _vp, _i32, _i32, _vp, _i64, _i64, _i64, _vp]),
    "lbq_q_push": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _i32, _i64, _i64, _vp, _i32, _i32, _i64, _i32, _vp]),
}

_lock = threading.Lock()
_lib = None


class LbqError(RuntimeError):
    """An lbq_* entry point returned a non-zero status."""


def load():
    """Load liblbq.so once and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: build it with `python -m lingbot_b200.build` "
                                  "(add --debug for the debug library; nvcc, sm_100a); there is no fallback "
                                  "implementation")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name, *args):
    """Call an lbq_* entry point that returns a status code; raise LbqError on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        msg = lib.lbq_last_error().decode(errors="replace")
        raise LbqError(f"{name} failed ({rc}): {msg}")
    return rc


def device_status(clear=True):
    """Read (and by default clear) the current device's status word: 0 unless a kernel's bounded
    wait gave up."""
    out = _i32(0)
    call("lbq_device_status", int(bool(clear)), ctypes.byref(out))
    return out.value
