"""CPU restatement of the reference's rowwise FP8 linear — TEST INFRASTRUCTURE ONLY (the checker of
lbq_fp8_quant_rows / lbq_fp8_gemm; imported by `tests/` only).

Parity status: the quantization is PINNED by `tests/golden/fp8_linear.npz`, which
`tests/golden/make_golden.py` generates by running the reference's own `FP8Linear`
(lingbot/layers/linear.py:10-31) on the CPU and recording the FP8 operands its forward hands to
`torch._scaled_mm`; `tests/test_fp8_golden.py` checks this file against them bit for bit (CPU rule),
and `tests/test_fp8_linear_gpu.py` checks the kernels against the reference's formulas run by torch on
the GPU (CUDA rule, see quant_rows). The GEMM is checked on the GPU against `torch._scaled_mm` itself
(the reference's call) and against `gemm` below, by tolerance: both accumulate in fp32 in their own
order. Citations are paths inside the reference.
"""
from __future__ import annotations

import torch

FMAX = 448.0          # torch.finfo(torch.float8_e4m3fn).max, linear.py:11


def quant_rows(x: torch.Tensor, device_rule="cuda"):
    """x [R, C] -> (e4m3 codes [R, C], fp32 scale [R, 1]): scale = max(|x| per row) / 448 in fp32,
    floored at 1e-12, codes = (x / scale) cast to e4m3 (linear.py:16-17 for weights, 24-25 for
    activations). torch evaluates the scalar division `amax / 448.0` differently per device: on CUDA,
    where the reference runs, as amax * fl(1/448) (a division by a Python scalar becomes a multiply by
    its fp32 reciprocal); on the CPU as a true division. device_rule "cuda" (the GPU kernels' rule) or
    "cpu" (the rule of the golden vectors, generated on the CPU); x / scale is a true division on both."""
    amax = x.abs().amax(dim=1, keepdim=True).float()
    if device_rule == "cuda":
        scale = amax * torch.tensor(1.0 / FMAX, dtype=torch.float32)
    else:
        scale = amax / FMAX
    scale = scale.clamp(min=1e-12)
    return (x.float() / scale).to(torch.float8_e4m3fn), scale


def gemm(qa, sa, qw, sw, bias=None):
    """y = (qa . qw^T) * sa * sw (+ bias), in float64 (the exact products and sums of the fp8 values),
    returned as float64 [M, N] (the GPU output is this rounded to bf16 after fp32 accumulation)."""
    y = qa.double() @ qw.double().t()
    y = y * sa.double().reshape(-1, 1) * sw.double().reshape(1, -1)
    if bias is not None:
        y = y + bias.to(torch.bfloat16).double().reshape(1, -1)
    return y
