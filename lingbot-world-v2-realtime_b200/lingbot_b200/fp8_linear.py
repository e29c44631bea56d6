"""FP8 linear layers on sm_100a — drop-in for the reference's rowwise `FP8Linear` and `convert_to_fp8`
(lingbot/layers/linear.py:10-31, 72-89).

Weights are quantized once, at construction, to e4m3 with one fp32 scale per output row; activations
are quantized per token on every call (lbq_fp8_quant_rows: the row's max |x| / 448, floored at 1e-12,
codes of x / scale). The GEMM is the tcgen05 kernel behind lbq_fp8_gemm: e4m3 x e4m3 with fp32
accumulation in tensor memory, both row scales and the bias applied in its epilogue, bf16 out — the
product the reference gets from torch._scaled_mm with rowwise scales. Only the rowwise mode is built;
the reference's MXFP8 mode (`LINGBOT_FP8=mx`) is not.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def quant_rows(x: torch.Tensor):
    """x [R, C] (bf16, fp16 or fp32, CUDA, unit column stride) -> (e4m3 codes [R, C], fp32 scales [R])."""
    if not x.is_cuda or x.dtype not in _DTYPES or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("quant_rows takes a 2-D CUDA bf16/fp16/fp32 tensor with unit column stride")
    r, c = x.shape
    q = torch.empty(r, c, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(r, dtype=torch.float32, device=x.device)
    _lib.call("lbq_fp8_quant_rows", _ptr(x), x.stride(0), _DTYPES[x.dtype], r, c, _ptr(q), q.stride(0), _ptr(s),
              _stream())
    return q, s


def gemm(qa, sa, qw, sw, bias=None, out=None):
    """y [M, N] bf16 = (qa [M, K] . qw [N, K]^T) * sa[m] * sw[n] (+ bias[n])."""
    m, k = qa.shape
    n = qw.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=qa.device)
    b = None if bias is None else bias.to(torch.bfloat16).contiguous()
    _lib.call("lbq_fp8_gemm", _ptr(qa), qa.stride(0), _ptr(sa), _ptr(qw), qw.stride(0), _ptr(sw),
              _ptr(b) if b is not None else None, m, n, k, _ptr(out), out.stride(0), 0, _stream())
    return out


class FP8Linear(torch.nn.Module):
    """`FP8Linear(lin)` of lingbot/layers/linear.py:10-31 on the GPU kernels: same quantization
    (bit-identical codes and scales), same product (fp32 accumulation, bf16 out)."""

    def __init__(self, lin: torch.nn.Linear):
        super().__init__()
        w = lin.weight.detach()
        if not w.is_cuda:
            raise ValueError("FP8Linear quantizes its weight on the GPU: move the layer to CUDA first")
        w8, ws = quant_rows(w.contiguous())
        self.register_buffer("w8", w8)                  # [N, K] e4m3
        self.register_buffer("w_scale", ws)             # [N] fp32
        self.bias = lin.bias
        self.in_features, self.out_features = lin.in_features, lin.out_features

    def forward(self, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x2.stride(-1) != 1 or x2.dtype not in _DTYPES:
            x2 = x2.contiguous()
        x8, xs = quant_rows(x2)
        y = gemm(x8, xs, self.w8, self.w_scale, self.bias)
        return y.reshape(*shape[:-1], y.shape[-1])


def convert_to_fp8(blocks, mx=False):
    """Swap the large nn.Linear layers inside `blocks` for FP8Linear, with the reference's selection rule
    (lingbot/layers/linear.py:72-89): in and out features >= 1024, in % 16 == 0, out % 16 == 0 — here
    out % 32 == 0 as well, which the DiT's 1536 / 8960 meet. Returns (fp8 count, linear count)."""
    if mx:
        raise NotImplementedError("the MXFP8 mode (LINGBOT_FP8=mx) is not built; use the rowwise mode")
    n_all, n_fp8 = 0, 0
    for parent in list(blocks.modules()):
        for name, m in list(parent.named_children()):
            if not isinstance(m, torch.nn.Linear):
                continue
            n_all += 1
            if m.in_features >= 1024 and m.out_features >= 1024 and m.in_features % 16 == 0 \
                    and m.out_features % 32 == 0:
                setattr(parent, name, FP8Linear(m))
                n_fp8 += 1
    return n_fp8, n_all
