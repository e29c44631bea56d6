"""The rowwise FP8 quantization restatement (oracle/fp8_linear.py) against the reference's own FP8Linear
(tests/golden/fp8_linear.npz from tests/golden/make_golden.py, run on the CPU): weights and
activations, codes and scales, bit for bit with torch's CPU division rule, including a zero row (scale
floored at 1e-12); and the CUDA rule differs from it only in the scale's last bit."""
import os

import numpy as np
import torch

from oracle import fp8_linear as F8

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "fp8_linear.npz")


def _bf16(bits):
    return torch.from_numpy(bits).view(torch.bfloat16)


def test_weight_quantization_matches_the_reference():
    g = np.load(GOLD)
    q, s = F8.quant_rows(_bf16(g["weight"]), device_rule="cpu")
    assert np.array_equal(q.view(torch.uint8).numpy(), g["w8"])
    assert np.array_equal(s.t().contiguous().numpy().view(np.int32), g["w_scale"].view(np.int32))
    assert np.array_equal(g["w8"], g["w8_seen"])


def test_activation_quantization_matches_the_reference():
    g = np.load(GOLD)
    q, s = F8.quant_rows(_bf16(g["x"]), device_rule="cpu")
    assert np.array_equal(q.view(torch.uint8).numpy(), g["x8"])
    assert np.array_equal(s.numpy().view(np.int32), g["x_scale"].view(np.int32))
    assert float(s[3]) == np.float32(1e-12)              # the zero row


def test_cuda_rule_is_the_reciprocal_multiply():
    g = np.load(GOLD)
    x = _bf16(g["x"])
    _, s_cpu = F8.quant_rows(x, device_rule="cpu")
    _, s_gpu = F8.quant_rows(x, device_rule="cuda")
    am = x.abs().amax(dim=1, keepdim=True).float()
    assert torch.equal(s_gpu, (am * np.float32(1.0 / 448.0)).clamp(min=1e-12))
    assert ((s_gpu.view(torch.int32) - s_cpu.view(torch.int32)).abs() <= 1).all()
