"""Torch-facing wrappers over the C ABI: buffer allocation, strides, streams.

Tensors are [B, L, H, 128] CUDA tensors ("NHD", the layout the reference's attention() receives),
bf16 — or fp16 on the drop-in path (quantize_qkv / attn_from_codes / sage_attn), the reference's
`dtype` choice. Every function launches on the current CUDA stream and never synchronises.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

HEAD_DIM = 128
NUM_SMS_B200 = 148


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


DTYPE_CODES = {torch.bfloat16: 0, torch.float16: 1}     # LBQ_DTYPE_BF16 / LBQ_DTYPE_F16


def _check_act(name, x, dtypes=(torch.bfloat16,)):
    if not x.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the quantized path has no CPU implementation)")
    if x.dtype not in dtypes:
        raise TypeError(f"{name} must be {' or '.join(str(d) for d in dtypes)}, got {x.dtype}")
    if x.dim() != 4 or x.shape[-1] != HEAD_DIM:
        raise ValueError(f"{name} must be [B, L, H, {HEAD_DIM}], got {tuple(x.shape)}")
    if x.stride(-1) != 1:
        raise ValueError(f"{name} must have unit channel stride")


def round_up(x, m):
    return (x + m - 1) // m * m


@dataclass
class QuantWindow:
    """Quantized Q and K/V of one attention call (layout in include/lbq.h)."""
    q_codes: torch.Tensor      # int8 [B, H, q_pad, 128]
    q_scale: torch.Tensor      # f32  [B, H, q_pad/32]
    k_codes: torch.Tensor      # int8 [S, B, H, seg_pad, 128]
    k_scale: torch.Tensor      # f32  [S, B, H, seg_pad/64]
    vt_codes: torch.Tensor     # uint8 (e4m3) [S, B, H, 128, seg_pad]
    v_scale: torch.Tensor      # f32  [B, H, 128]
    km: torch.Tensor           # [B, H, 128] in the activations' dtype
    q_len: int
    kv_len: int
    seg_len: int
    num_segments: int = 1
    dtype: torch.dtype = torch.bfloat16   # of the activations, and of attn_from_codes' output


def alloc_q(batch, heads, q_len, device):
    q_pad = round_up(q_len, 128)
    return (torch.empty(batch, heads, q_pad, HEAD_DIM, dtype=torch.int8, device=device),
            torch.empty(batch, heads, q_pad // 32, dtype=torch.float32, device=device))


def alloc_kv(batch, heads, seg_len, num_segments, device, dtype=torch.bfloat16):
    seg_pad = round_up(seg_len, 128)
    return (torch.empty(num_segments, batch, heads, seg_pad, HEAD_DIM, dtype=torch.int8, device=device),
            torch.empty(num_segments, batch, heads, seg_pad // 64, dtype=torch.float32, device=device),
            torch.empty(num_segments, batch, heads, HEAD_DIM, seg_pad, dtype=torch.uint8, device=device),
            torch.empty(batch, heads, HEAD_DIM, dtype=torch.float32, device=device),
            torch.empty(batch, heads, HEAD_DIM, dtype=dtype, device=device))


def quantize_qkv(q, k, v) -> QuantWindow:
    """Sage's per-call quantization of (q, k, v): Q per 32-token group, K mean-smoothed per 64-token
    block, V per channel e4m3 (lbq_quant_qkv). q, k, v: all bf16 or all fp16."""
    for n, x in (("q", q), ("k", k), ("v", v)):
        _check_act(n, x, tuple(DTYPE_CODES))
    if not q.dtype == k.dtype == v.dtype:
        raise TypeError(f"q, k, v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    b, lq, h, _ = q.shape
    lk = k.shape[1]
    if k.shape != v.shape or k.shape[0] != b or k.shape[2] != h:
        raise ValueError(f"k/v shapes {tuple(k.shape)} / {tuple(v.shape)} do not match q {tuple(q.shape)}")
    dev = q.device
    q_codes, q_scale = alloc_q(b, h, lq, dev)
    k_codes, k_scale, vt_codes, v_scale, km = alloc_kv(b, h, lk, 1, dev, q.dtype)
    lib = _lib.load()
    ws_bytes = lib.lbq_quant_qkv_workspace(b, h, lk)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.call("lbq_quant_qkv", _ptr(q), *q.stride()[:3], lq, _ptr(k), *k.stride()[:3], _ptr(v), *v.stride()[:3],
              lk, b, h, _ptr(q_codes), _ptr(q_scale), _ptr(k_codes), _ptr(k_scale), _ptr(vt_codes),
              _ptr(v_scale), _ptr(km), _ptr(ws), ws_bytes, DTYPE_CODES[q.dtype], _stream())
    return QuantWindow(q_codes, q_scale, k_codes, k_scale, vt_codes, v_scale, km, lq, lk, lk, 1, q.dtype)


def pick_splits(batch, heads, q_len, kv_len, num_sms=NUM_SMS_B200):
    """Split the key range when the grid cannot fill the SMs. A CTA of the attention kernel holds a
    pair of 128-row Q tiles and occupies a whole SM, so the split count is the largest one that keeps
    the grid within one wave (no tail), and never makes a split shorter than 8 key tiles."""
    ctas = ((round_up(q_len, 128) // 128 + 1) // 2) * batch * heads
    tiles = (kv_len + 127) // 128
    if ctas >= num_sms:
        return 1
    return max(1, min(num_sms // ctas, tiles // 8))


def attn_from_codes(w: QuantWindow, sm_scale=None, out=None, num_splits=None, is_causal=False):
    """Attention over a quantized window -> [B, q_len, H, 128] in w.dtype (lbq_attn_fwd [+ combine]).
    is_causal=True is refused by the C ABI (LBQ_ERR_UNSUPPORTED -> RuntimeError)."""
    b, h = w.q_codes.shape[0], w.q_codes.shape[1]
    dev = w.q_codes.device
    if out is None:
        out = torch.empty(b, w.q_len, h, HEAD_DIM, dtype=w.dtype, device=dev)
    _check_act("out", out, (w.dtype,))
    dt = DTYPE_CODES[w.dtype]
    if num_splits is None:
        num_splits = pick_splits(b, h, w.q_len, w.kv_len)
    q_pad = w.q_codes.shape[2]
    o_part = ml_part = None
    if num_splits > 1:
        o_part = torch.empty(num_splits, b * h, q_pad, HEAD_DIM, dtype=torch.float32, device=dev)
        ml_part = torch.empty(num_splits, b * h, q_pad, 2, dtype=torch.float32, device=dev)
    used = ctypes.c_int(1)
    _lib.call("lbq_attn_fwd", _ptr(w.q_codes), _ptr(w.q_scale), w.q_len, _ptr(w.k_codes), _ptr(w.k_scale),
              _ptr(w.vt_codes), _ptr(w.v_scale), w.kv_len, w.num_segments, w.seg_len, b, h,
              float(sm_scale or 0.0), int(bool(is_causal)), _ptr(out), *out.stride()[:3], num_splits,
              _ptr(o_part) if o_part is not None else None, _ptr(ml_part) if ml_part is not None else None,
              ctypes.byref(used), dt, _stream())
    if used.value > 1:
        _lib.call("lbq_splitkv_combine", _ptr(o_part), _ptr(ml_part), used.value, _ptr(w.v_scale), b, h, w.q_len,
                  _ptr(out), *out.stride()[:3], dt, _stream())
    return out


def sage_attn(q, k, v, sm_scale=None, num_splits=None, out=None, is_causal=False):
    """`sageattn(q, k, v, tensor_layout="NHD", is_causal, sm_scale=sm_scale)` on sm_100a, bf16 or fp16
    in and out; is_causal=True raises (the kernel has no causal mask: LBQ_ERR_UNSUPPORTED)."""
    w = quantize_qkv(q, k, v)
    return attn_from_codes(w, sm_scale=sm_scale, out=out, num_splits=num_splits, is_causal=is_causal)
