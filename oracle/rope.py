"""CPU restatement of the reference's RoPE — TEST INFRASTRUCTURE ONLY (the checker of lbq_rope_quant_q
and lbq_cache_write's roped K; imported by `tests/` only).

Parity status: PINNED by `tests/golden/rope_grid2x4x6.npz`, which `tests/golden/make_golden.py` generates by
running the reference's own `rope_params` (reference/wan/modules/model.py:29-36), `causal_rope_freqs`
and `causal_rope_apply` (lingbot/models/lingbot_world/transformer.py:53-76, 134-146);
`tests/test_rope_golden.py` checks this file against them bit for bit. Citations are paths inside the
reference project.
"""
from __future__ import annotations

import torch


def rope_angles(max_seq_len: int, dim: int, theta: float = 10000.0) -> torch.Tensor:
    """[max_seq_len, dim/2] float64 angles p * theta^(-2i/dim) (wan/modules/model.py:29-36 builds the
    polar table exp(i * angle) from these)."""
    inv = 1.0 / torch.pow(torch.tensor(theta, dtype=torch.float64),
                          torch.arange(0, dim, 2, dtype=torch.float64) / dim)
    return torch.outer(torch.arange(max_seq_len, dtype=torch.float64), inv)


def freqs_table(head_dim: int = 128) -> torch.Tensor:
    """The DiT's [1024, head_dim/2, 2] (cos, sin) table: frame, height and width bands of
    head_dim - 4*(head_dim//6), 2*(head_dim//6), 2*(head_dim//6) channels (transformer.py:553-558)."""
    d = head_dim
    parts = [rope_angles(1024, d - 4 * (d // 6)), rope_angles(1024, 2 * (d // 6)), rope_angles(1024, 2 * (d // 6))]
    ang = torch.cat(parts, dim=1)
    polar = torch.polar(torch.ones_like(ang), ang)
    return torch.view_as_real(polar)


def rope_tables(grid_sizes, freqs: torch.Tensor, start_frame: int = 0):
    """(cos, sin), each [B, L, 64] float64, for tokens laid out frame-major then row then column
    (transformer.py:53-76): channel pair i of token (f, y, x) takes the frame band's angle of
    start_frame + f, the height band's of y or the width band's of x."""
    c = freqs.shape[1]
    nf = c - 2 * (c // 3)
    bands = (freqs[:, :nf], freqs[:, nf:nf + c // 3], freqs[:, nf + c // 3:])
    out = []
    for f, h, w in grid_sizes:
        fr = bands[0][start_frame:start_frame + f].reshape(f, 1, 1, -1, 2).expand(f, h, w, -1, -1)
        hr = bands[1][:h].reshape(1, h, 1, -1, 2).expand(f, h, w, -1, -1)
        wr = bands[2][:w].reshape(1, 1, w, -1, 2).expand(f, h, w, -1, -1)
        out.append(torch.cat([fr, hr, wr], dim=-2).reshape(f * h * w, -1, 2))
    t = torch.stack(out)
    return t[..., 0].contiguous(), t[..., 1].contiguous()


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, L, H, D] (bf16) rotated per channel pair (2i, 2i+1) in float64,
    (xr cos - xi sin, xr sin + xi cos), each product and sum rounded in float64, cast back to x's dtype
    (transformer.py:142-146). cos / sin: [B, L, D/2]."""
    xd = x.to(torch.float64).unflatten(-1, (-1, 2))
    xr, xi = xd[..., 0], xd[..., 1]
    c, s = cos[:, :, None, :], sin[:, :, None, :]
    re = xr * c - xi * s
    im = xr * s + xi * c
    return torch.stack([re, im], dim=-1).flatten(-2).to(x.dtype)
