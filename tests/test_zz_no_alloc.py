"""lbq_quant_qkv_static — the quantizer entry point for callers that cannot give the library device
memory (a runtime whose device memory pool is fixed and owned elsewhere, or an FFI binding with no way
to pass a workspace) — must produce exactly what lbq_quant_qkv produces with a caller workspace.

Called twice in a row on different inputs: the static scratch is shared by every call and keeps the
previous call's contents, so the second call also checks that nothing stale leaks into it. This file
is collected last (test_zz_*) so that a run stopping at its first failure has run everything else.
"""
import ctypes

import pytest
import torch

from tests._gpu import make_qkv

pytestmark = pytest.mark.gpu


def _buffers(b, h, lq, lk, dev):
    from lingbot_b200 import ops
    qc, qs = ops.alloc_q(b, h, lq, dev)
    kc, ks, vt, vs, km = ops.alloc_kv(b, h, lk, 1, dev)
    for t in (qc, qs, kc, ks, vt, vs, km):
        t.zero_()
    return dict(q_codes=qc, q_scale=qs, k_codes=kc, k_scale=ks, vt_codes=vt, v_scale=vs, km=km)


def _outs(bufs):
    return [bufs[n] for n in ("q_codes", "q_scale", "k_codes", "k_scale", "vt_codes", "v_scale", "km")]


def _call(name, q, k, v, bufs, ws=None):
    from lingbot_b200 import _lib
    from lingbot_b200.ops import _ptr, _stream
    b, lq, h, _ = q.shape
    lk = k.shape[1]
    args = [_ptr(q), *q.stride()[:3], lq, _ptr(k), *k.stride()[:3], _ptr(v), *v.stride()[:3], lk, b, h,
            *[_ptr(t) for t in _outs(bufs)]]
    if ws is not None:
        args += [_ptr(ws), ws.numel()]
    _lib.call(name, *args, 0, _stream())                    # LBQ_DTYPE_BF16


@pytest.mark.parametrize("shape", [(1, 12, 6032, 12064), (2, 3, 513, 4097)], ids=["config1", "batch2-odd"])
def test_static_scratch_matches_workspace_entry_point_twice(shape):
    from lingbot_b200 import _lib
    b, h, lq, lk = shape
    dev = torch.device("cuda")
    lib = _lib.load()
    for seed in (21, 22):                                    # two calls in a row, different inputs
        q, k, v = make_qkv(seed, b, h, lq, lk)
        ref = _buffers(b, h, lq, lk, dev)
        ws = torch.empty(lib.lbq_quant_qkv_workspace(b, h, lk), dtype=torch.uint8, device=dev)
        _call("lbq_quant_qkv", q, k, v, ref, ws)
        got = _buffers(b, h, lq, lk, dev)
        _call("lbq_quant_qkv_static", q, k, v, got)
        torch.cuda.synchronize()
        for name in ref:
            assert torch.equal(got[name], ref[name]), f"{name} differs (call with seed {seed})"


def test_static_scratch_rejects_windows_past_its_capacity():
    """batch 1 x 12 heads fits 58176 keys in the 16 MiB scratch; one more 64-token block does not."""
    from lingbot_b200 import _lib
    lib = _lib.load()
    ok = lib.lbq_quant_qkv_workspace(1, 12, 58176)
    too_big = lib.lbq_quant_qkv_workspace(1, 12, 58177)
    assert ok <= (16 << 20) < too_big
    null = ctypes.c_void_p(0)
    rc = lib.lbq_quant_qkv_static(null, 0, 0, 0, 1, null, 0, 0, 0, null, 0, 0, 0, 58177, 1, 12,
                                  null, null, null, null, null, null, null, 0, null)
    assert rc == 1
    assert b"static" in lib.lbq_last_error() and b"workspace" in lib.lbq_last_error()
