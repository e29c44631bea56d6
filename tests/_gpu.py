"""Helpers for the GPU parity tests: unpack the CUDA path's code buffers into the oracle's layout."""
import torch


def q_codes_nhd(w):
    """[B, H, q_pad, 128] -> [B, q_len, H, 128]"""
    return w.q_codes[:, :, :w.q_len].permute(0, 2, 1, 3).cpu()


def k_codes_nhd(w):
    """[S, B, H, seg_pad, 128] (one segment) -> [B, kv_len, H, 128]"""
    return w.k_codes[0][:, :, :w.kv_len].permute(0, 2, 1, 3).cpu()


def k_scale_ref(w):
    """[S, B, H, seg_pad/64] -> [B, H, ceil(kv/64)] (the reference's block count)"""
    nb = (w.kv_len + 63) // 64
    return w.k_scale[0][:, :, :nb].cpu()


def v_codes_nhd(w):
    """[S, B, H, 128, seg_pad] -> [B, kv_len, H, 128]"""
    return w.vt_codes[0][:, :, :, :w.kv_len].permute(0, 3, 1, 2).cpu()


def bits(t):
    return t.contiguous().view(torch.int32) if t.dtype == torch.float32 else t


def make_qkv(seed, b, h, lq, lk, koff=3.0, outlier=None, device="cuda"):
    """Seeded [B, L, H, 128] bf16 inputs: N(0,1), K + per-channel N(0, koff) offset, optional
    outlier channels (x20)."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, lq, h, 128, generator=g)
    k = torch.randn(b, lk, h, 128, generator=g)
    v = torch.randn(b, lk, h, 128, generator=g)
    if koff:
        k = k + torch.randn(b, 1, h, 128, generator=g) * koff
    if outlier == "four":
        k[..., :4] *= 20
    return tuple(x.bfloat16().to(device) for x in (q, k, v))
