"""Drop-in for the reference's attention operator (lingbot/layers/attention.py:27-40).

`attention(q, k, v, ...)` keeps the reference's signature. The plain batched call (no q_lens /
k_lens, no dropout, not causal) — the only way the causal DiT calls it
(models/lingbot_world/transformer.py:225) — runs the B200 quantized kernels (INT8 QK^T, FP8 PV,
SageAttention-2 semantics) on q/k/v cast to `dtype` (bf16 by default, or fp16), as the reference
casts before Sage (lingbot/layers/attention.py:30-36). Every other call takes the reference's non-Sage
branch, which is the paper's attention (wan/modules/attention.py:132-178); here that is torch's SDPA
on the GPU. That includes causal=True, which the reference would hand to Sage with is_causal: the
quantized kernel has no causal mask and its C ABI refuses one (LBQ_ERR_UNSUPPORTED).
The quantized path is registered as the custom op `lbq::sage_attn` (with a fake implementation) so
torch.compile keeps the DiT in one graph, as the reference relied on for `sageattn`.

`flash_attention(q, k, v, k_lens=None)` is the reference's cross-attention entry
(lingbot/layers/attention.py:16-20, called at models/lingbot_world/transformer.py:272 with
k_lens=None, transformer.py:658). Like the reference it is not quantized by default. With
`LBQ_CROSS_ATTN=sage` in the environment (or `set_cross_attention("sage")`), its plain calls run
through the same quantized kernels: q of the chunk against the 512 text keys.
"""
import os

import torch
import torch.nn.functional as F

from . import ops

__all__ = ["attention", "flash_attention", "set_cross_attention"]


@torch.library.custom_op("lbq::sage_attn", mutates_args=())
def sage_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float) -> torch.Tensor:
    """q/k/v [B, L, H, 128], all bf16 or all fp16 -> [B, Lq, H, 128] in that dtype."""
    return ops.sage_attn(q, k, v, sm_scale=sm_scale if sm_scale > 0 else None)


@sage_attn.register_fake
def _(q, k, v, sm_scale):
    return torch.empty_like(q)


def _paper_attention(q, k, v, q_lens=None, k_lens=None, dropout_p=0., softmax_scale=None, causal=False,
                     dtype=torch.bfloat16):
    """The reference's non-Sage branch: padded-batch attention with optional key lengths."""
    out_dtype = q.dtype
    lq = q.shape[1]
    qh, kh, vh = (x.to(dtype).transpose(1, 2) for x in (q, k, v))
    mask = None
    if k_lens is not None:
        keep = torch.arange(k.shape[1], device=k.device)[None, :] < k_lens.to(k.device)[:, None]
        mask = keep[:, None, None, :]
    o = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, dropout_p=dropout_p,
                                       is_causal=causal and mask is None, scale=softmax_scale)
    o = o.transpose(1, 2)
    if q_lens is not None:
        valid = torch.arange(lq, device=q.device)[None, :] < q_lens.to(q.device)[:, None]
        o = o * valid[:, :, None, None]
    return o.to(out_dtype)


_CROSS_MODES = ("paper", "sage")
_cross_mode = os.environ.get("LBQ_CROSS_ATTN", "paper")
if _cross_mode not in _CROSS_MODES:
    raise ValueError(f"LBQ_CROSS_ATTN={_cross_mode!r}: expected one of {_CROSS_MODES}")


def set_cross_attention(mode):
    """Route flash_attention's plain calls to the paper's attention ("paper", the default, as the
    reference does) or to the quantized kernels ("sage")."""
    global _cross_mode
    if mode not in _CROSS_MODES:
        raise ValueError(f"cross-attention mode {mode!r}: expected one of {_CROSS_MODES}")
    _cross_mode = mode


def flash_attention(q, k, v, k_lens=None, **kw):
    """The reference's cross-attention entry (lingbot/layers/attention.py:16-20). Quantized only in
    the "sage" cross-attention mode and only for plain calls (no k_lens, no dropout, not causal)."""
    kw.pop("fa_version", None)
    kw.pop("q_scale", None)
    kw.pop("window_size", None)
    kw.pop("deterministic", None)
    if (_cross_mode == "sage" and k_lens is None and kw.get("q_lens") is None and not kw.get("dropout_p")
            and not kw.get("causal")):
        scale = kw.get("softmax_scale")
        out_dtype = q.dtype
        x = sage_attn(q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16),
                      float(scale) if scale else 0.0)
        return x.to(out_dtype)
    return _paper_attention(q, k, v, k_lens=k_lens, **kw)


def attention(q, k, v, q_lens=None, k_lens=None, dropout_p=0., softmax_scale=None, q_scale=None,
              causal=False, window_size=(-1, -1), deterministic=False, dtype=None, fa_version=None):
    dtype = torch.bfloat16 if dtype is None else dtype
    if q_lens is None and k_lens is None and dropout_p == 0. and not causal:
        if dtype not in ops.DTYPE_CODES:
            raise TypeError(f"attention(dtype={dtype}): the quantized kernels take bfloat16 or float16")
        # q/k/v are [B, L, H, D] ("NHD"); Lq != Lk is fine without a mask (attention.py:32-36)
        out_dtype = q.dtype
        x = sage_attn(q.to(dtype), k.to(dtype), v.to(dtype), float(softmax_scale) if softmax_scale else 0.0)
        return x.to(out_dtype)
    return _paper_attention(q, k, v, q_lens=q_lens, k_lens=k_lens, dropout_p=dropout_p,
                            softmax_scale=softmax_scale, causal=causal, dtype=dtype)
