"""CPU restatement of SageAttention-2 semantics as the reference uses them — TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path. It is imported by `tests/`, by
`__graft_entry__.smoke()` and by the CPU legs of `bench.py`; the product never calls it.

Parity status:
  * Quantizers (Q per-warp int8, K mean-smoothed per-64-token int8, V per-channel e4m3) are
    PINNED: `tests/golden/make_golden.py` runs the reference's own torch quantizers
    (`experiments/modules/sage_kvq.py:57-75`) in the build container and commits their outputs;
    `tests/test_oracle_golden.py` checks this file against them bit for bit.
  * The attention kernel emulation (`attn_from_codes`) follows the kernel semantics the reference
    documents (`experiments/bench_attn/splitkv/README.md:51-69`,
    `experiments/bench_attn/h2_tiles/cfg_fixedmax.patch:90-93`, `phi_calib.md:12-13`,
    `sage_kvq.py:15-19`). SageAttention itself is not vendored and has no CPU build, so this part
    is checked by tolerance (cosine / max-abs), not bits: parity of the attention output is
    unpinned by golden vectors, as in the reference, whose own tests replace Sage by SDPA.

All citations are paths inside the reference project.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

# sage_kvq.py:29-35 — tile constants of the sm89 kernel the reference calls
BLK_K, BLK_Q, WARP_Q = 64, 128, 32
# sage_kvq.py:30-31 / sage_preq.py:66 — V scale ceiling for the fp32+fp16 PV accumulator
V_SCALE_MAX = 2.25
# splitkv/README.md:58, cfg_fixedmax.patch:13 — log2-domain offset that puts the row max of P at 448
S_FP8_OFFSET = 8.807
LOG2E = 1.4426950408889634
# sage_kvq.py:34-35 — Sage's V layout permutes every 16 tokens like this
V_PERM = [0, 1, 8, 9, 2, 3, 10, 11, 4, 5, 12, 13, 6, 7, 14, 15]


def quant_int8(x: torch.Tensor, blk: int, pad_to: int, mean: torch.Tensor | None = None):
    """Restates `sage_kvq._quant_int8` (sage_kvq.py:57-66) and Sage's QuantInt8Kernel.

    x [B, n, H, D] (bf16) -> (codes int8 [B, n, H, D], scale f32 [B, H, ceil(n/pad_to)*pad_to/blk]).
    Tokens past n count as zero (after the mean is subtracted). Codes are
    round-half-even(x * (127/amax)) saturated to [-128, 127] in fp32; scale = amax/127 with
    amax floored at 1e-7. The reference writes `127.0 / amax`, which torch evaluates as
    reciprocal(amax) * 127 (two fp32 roundings, not one division); `amax / 127.0` is a true
    fp32 division. Both are reproduced exactly here and in the CUDA kernels.
    """
    b, n, h, d = x.shape
    xf = x.float() if mean is None else x.float() - mean.float()
    lp = (n + pad_to - 1) // pad_to * pad_to
    xf = F.pad(xf, (0, 0, 0, 0, 0, lp - n)).view(b, lp // blk, blk, h, d)
    amax = xf.abs().amax(dim=(2, 4)).clamp_min(1e-7)
    inv = torch.reciprocal(amax) * 127.0               # == torch's `127.0 / amax`
    xq = (xf * inv[:, :, None, :, None]).round().clamp(-128, 127).to(torch.int8)
    scale = (amax / 127.0).transpose(1, 2).contiguous()
    return xq.view(b, lp, h, d)[:, :n], scale


def quant_q(q: torch.Tensor):
    """Q: one scale per (batch, head, 32-token group), Lq padded to 128 (per_warp_int8 with
    BLKQ=128, WARPQ=32; call at sage_preq.py:116, restated at sage_kvq.py:104)."""
    return quant_int8(q, WARP_Q, BLK_Q)


def k_mean(k: torch.Tensor) -> torch.Tensor:
    """km = mean of K over the window's tokens, rounded to K's dtype (sage_preq.py:115,
    `k.mean(dim=1, keepdim=True)`). The sum is taken in float64, i.e. the exact mean of the bf16
    inputs rounded once; torch's own fp32 reduction can differ from it by one bf16 ulp at a
    rounding boundary (tests allow that one ulp against the reference and demand bits here)."""
    return k.double().mean(dim=1, keepdim=True).to(k.dtype)


def quant_k(k: torch.Tensor, km: torch.Tensor):
    """K: subtract km, one scale per (batch, head, 64-token block) (sage_preq.py:116 with
    BLKK=64; sage_kvq.py:85)."""
    return quant_int8(k, BLK_K, BLK_K, km)


def v_amax(v: torch.Tensor) -> torch.Tensor:
    """Per-(batch, head, channel) max |v| over the window (sage_preq.py:47-63 min/max table,
    sage_kvq.py:97 without the experimental V_MARGIN). Zero padding never raises it."""
    return v.float().abs().amax(dim=1)


def e4m3_rn_satfinite(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> e4m3 code (uint8), round-to-nearest-even, saturating to +-448 like the
    `cvt.rn.satfinite.e4m3x2.f32` the CUDA kernels use (torch's cast alone turns >=464 into NaN)."""
    return x.clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_to_float(codes: torch.Tensor) -> torch.Tensor:
    return codes.view(torch.float8_e4m3fn).float()


def quant_v(v: torch.Tensor, amax: torch.Tensor):
    """V: e4m3 codes of v * (2.25/amax) per (batch, head, channel), clamped to +-2.25
    (sage_kvq.py:69-75, sage_preq.py:54,67-77). Returns codes in the natural token order
    [B, n, H, D] (uint8) and v_scale = amax/2.25 [B, H, D]. Sage stores the same codes
    transposed and permuted (`sage_layout`); the CUDA path stores them as V^T per head."""
    recp = torch.reciprocal(amax) * V_SCALE_MAX        # == torch's `V_SCALE_MAX / v_amax`
    x = v.float() * recp[:, None]
    codes = x.clamp(-V_SCALE_MAX, V_SCALE_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    return codes, amax / V_SCALE_MAX


def sage_layout(v_codes: torch.Tensor) -> torch.Tensor:
    """Natural-order V codes [B, n, H, D] (n % 16 == 0) -> Sage's [B, D, H, n] with the 16-token
    permutation (sage_kvq.py:73-75)."""
    b, n, h, d = v_codes.shape
    vp = v_codes.view(b, n // 16, 16, h, d)[:, :, V_PERM].reshape(b, n, h, d)
    return vp.permute(0, 3, 2, 1)


def quantize_qkv(q, k, v):
    """The quantization half of `sageattn(q, k, v, "NHD")` as the reference drives it
    (attention.py:34 -> per_warp_int8 + per_channel_fp8, sage_preq.py:115-124)."""
    qc, qs = quant_q(q)
    km = k_mean(k)
    kc, ks = quant_k(k, km)
    am = v_amax(v)
    vc, vs = quant_v(v, am)
    return dict(q_codes=qc, q_scale=qs, km=km, k_codes=kc, k_scale=ks, v_codes=vc, v_scale=vs,
                v_amax=am)


def attn_from_codes(q_codes, q_scale, k_codes, k_scale, v_codes, v_scale, sm_scale=None,
                    pv_accum="fp16", rows=None, heads=None, splits=1, key_ranges=None,
                    partial_fp16=False, ambiguous=None):
    """Torch emulation of Sage's `qk_int8_sv_f8_accum_f16_fuse_v_scale_attn_inst_buf` (the call at
    sage_preq.py:126-127 / sage_kvq.py:107-110), non-causal, per-warp Q granularity, with the kernel's
    own fp32 arithmetic order.

    The loop runs over 64-key tiles (CTA_K = 64, sage_kvq.py:29) in order. For a row with Q scale
    q_s (its 32-row group) and a tile with K scale k_s (its 64-token block), S = q_i8 . k_i8 (exact
    int32), and with sm = fl(sm_scale * log2 e):
      main tiles    c = fl(sm * fl(q_s * k_s))       the per-tile scale upstream passes to update_mdo
                    m_t = fma(max_j S_j, c, -8.807)   (cfg_condrescale.patch:20, cfg_fusedsoftmax.patch:127)
                    x_j = fma(S_j, c, -m)             (cfg_fusedsoftmax.patch:157)
      last 2 tiles  r_j = fl(S_j * fl(q_s * k_s))    upstream's last two iterations call update_mdo with
                    m_t = fma(max_j r_j, sm, -8.807)  `original_sm_scale` (cfg_fixedmax.patch:307,329), i.e.
                    x_j = fma(r_j, sm, -m)            on scores that already carry the dequant scale
      m     = max(m_prev, m_t)                        (m starts at -inf: upstream's -5e6 with d = 1 is
      alpha = exp2(m_prev - m)                         cleared by the first alpha = 0)
      P_j   = exp2(x_j)                               (fp32, <= 448: the row max lands on 2^8.807)
      d     = d * alpha + sum_j P_j                   (fp32 P, before the e4m3 rounding)
      O     = O * alpha + e4m3(P) @ e4m3(V)           (fp16 inside a tile in 32-key steps when
                                                       pv_accum == "fp16", the "inst buf"; else fp32)
      out   = O / d * v_scale                         (splitkv/README.md:51-69)
    Each fma is evaluated exactly in float64 and rounded once to float32 (the products S * c fit in
    45 bits). `m` is in the log2 domain and includes -8.807 and the dequant scale
    (splitkv/README.md:58).

    Returns fp32 [B, Lq, H, D]. `rows` / `heads` restrict the computation to a subset (query rows
    are independent, so the subset equals the same rows of the full result).
    `splits` > 1 emulates split-KV (splitkv/README.md:36-69) as the CUDA path cuts it: the 128-key
    tiles are cut into `splits` contiguous ranges (ceil division, empty ranges dropped), each runs the
    loop above from a fresh running max (its own last two tiles included), and the partials merge as
    out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) d_s.
    `key_ranges` replaces the split ranges with the key-range sequence split: one partial per rank,
    each a list of (lo, hi) key ranges (lo a multiple of 64) that the rank's loop runs through in
    order with one running max (its memory tiles, then its chunk share). With `partial_fp16` each
    partial travels as fp16(O_s / d_s) with (m_s, d_s), and the merge is
    out = sum_s w_s fp16(O_s / d_s) / sum_s w_s with w_s = 2^(m_s - M) d_s.
    With `ambiguous` (a bool tensor [B, Lq, H], set in place), a row is marked when the P of the row
    that lie within the GPU kernel's own error of an e4m3 rounding midpoint could, all flipping one e4m3
    step the same way, move the row's output by more than AMBIGUOUS_IMPACT: their e4m3 values depend on
    the last bits of the exp2 implementation (ex2.approx on the GPU, a correctly rounded exp2 here), and
    outside the last two tiles also on the kernel's folded exp2 argument and polynomial exp2
    (bulk_rel_err).
    """
    b, lq, h, d = q_codes.shape
    lk = k_codes.shape[1]
    if sm_scale is None:
        sm_scale = d ** -0.5
    # fl(fl(sm_scale) * fl(log2 e)): the fp32 product the kernel forms from its float argument
    sm_log2 = torch.tensor(sm_scale, dtype=torch.float32) * torch.tensor(LOG2E, dtype=torch.float32)
    rows = torch.arange(lq) if rows is None else torch.as_tensor(rows)
    heads = range(h) if heads is None else heads
    out = torch.zeros(b, lq, h, d, dtype=torch.float32)
    vq_all = e4m3_to_float(v_codes)                                    # [B, Lk, H, D]
    n128 = (lk + 127) // 128
    per = (n128 + splits - 1) // splits
    partials = [[(s0 * 128, min(lk, (s0 + per) * 128))] for s0 in range(0, n128, per)]
    if key_ranges is not None:
        partials = [[(lo, hi_) for lo, hi_ in pieces if hi_ > lo] for pieces in key_ranges]
        partials = [p for p in partials if p]
    for bi in range(b):
        for hi in heads:
            qf = q_codes[bi, rows, hi].float()                          # [R, D]
            qs = q_scale[bi, hi][rows // WARP_Q]                         # [R]
            kf = k_codes[bi, :, hi].float()                             # [Lk, D]
            vf = vq_all[bi, :, hi]                                       # [Lk, D]
            parts, ambs = [], []
            for pieces in partials:
                tiles = [(t0, min(t0 + BLK_K, hi_)) for lo, hi_ in pieces for t0 in range(lo, hi_, BLK_K)]
                state = None
                amb = None if ambiguous is None else torch.zeros(qf.shape[0], dtype=torch.float64)
                for i, (t0, t1) in enumerate(tiles):
                    state = _attn_tile(qf, qs, kf, vf, k_scale[bi, hi][t0 // BLK_K], t0, t1, pv_accum, sm_log2,
                                       state, tail=i >= len(tiles) - 2, amb=amb)
                parts.append(state)
                ambs.append(amb)
            mx = torch.stack([p[0] for p in parts]).max(dim=0).values
            acc = torch.zeros(qf.shape[0], d)
            dsum = torch.zeros(qf.shape[0])
            for m_s, d_s, o_s in parts:
                w = torch.exp2(m_s - mx)
                if partial_fp16:
                    o_s = (o_s / d_s[:, None]).half().float() * d_s[:, None]
                acc += w[:, None] * o_s
                dsum += w * d_s
            o = acc * (1.0 / dsum)[:, None] * v_scale[bi, hi][None, :]
            out[bi, rows, hi] = o
            if ambiguous is not None:
                # a flip of one e4m3 step 2^a (a in the log2 units of the partial's running max m_s, see
                # _attn_tile) moves the output by at most 2^(a - M) * max|V| / D; `amb` sums 2^a
                vmax = float(v_scale[bi, hi].max()) * V_SCALE_MAX
                total = sum(a_sum * torch.exp2(-mx.double()) for a_sum in ambs)
                ambiguous[bi, rows, hi] |= total * vmax / dsum.double() > AMBIGUOUS_IMPACT
    return out


def _fma32(a, b, c):
    """fp32 fma(a, b, c) for float32 tensors: the exact value in float64 (a * b has at most 48
    significant bits here), rounded once to float32."""
    return (a.double() * b.double() + c.double()).float()


# ex2.approx.ftz.f32's relative error is about 2^-22 (2 ulp); a P within 2^-20 of an e4m3 rounding
# midpoint (a margin of 4x) may round either way on the GPU. A row is ambiguous when one-step flips of
# all such P of the row could together move an output by more than AMBIGUOUS_IMPACT (half the max-abs
# tolerance of 2e-2, so that a row held to the tolerance keeps half of it for every other error).
EXP2_REL_ERR = 2.0 ** -20
AMBIGUOUS_IMPACT = 1e-2
# The GPU kernel's bulk tiles (all but the last two 64-key tiles of a pass) evaluate the exp2 argument as
# fma(1.5*2^23 + S, c, fl(-1.5*2^23 * c - m)) where fl(1.5*2^23 * c) < FOLD_MAX (for both 64-key tiles of
# a 128-key tile; taking the bound per 64-key tile here only widens the window), and there take some
# keys' exp2 from a degree-3 polynomial (max relative error 7.48e-5, measured on a 2e6-point grid of
# [-0.5, 0.5], plus fp32 rounding).
KERNEL_MAGIC = 12582912.0
FOLD_MAX = 4096.0
POLY_REL_ERR = 7.6e-5


def _ulp32(v: torch.Tensor) -> torch.Tensor:
    """ulp of float32 values (0 -> the smallest normal's)."""
    _, ex = torch.frexp(v.float().abs())
    return torch.exp2((ex - 24).clamp(min=-149).double())


def bulk_rel_err(x: torch.Tensor, scale: torch.Tensor, m_new: torch.Tensor) -> torch.Tensor:
    """Bound on the relative error of the GPU kernel's P in a bulk tile, per element: ex2, plus ln 2
    times one ulp of x; and where the kernel folds the magic bias into the argument (and then takes some
    keys' exp2 from the polynomial), the polynomial's error and ln 2 times half an ulp of the folded
    constant fl(-1.5*2^23 * c - m)."""
    fold = (torch.tensor(KERNEL_MAGIC, dtype=torch.float32) * scale.float()) < FOLD_MAX
    b = _fma32(torch.full_like(scale, -KERNEL_MAGIC), scale, -m_new)
    zero = torch.zeros_like(b, dtype=torch.float64)
    extra = torch.where(fold, POLY_REL_ERR + math.log(2.0) * 0.5 * _ulp32(b), zero)
    return EXP2_REL_ERR + extra[:, None] + math.log(2.0) * _ulp32(x)


def _ambiguous_steps(p: torch.Tensor, m: torch.Tensor, rel_err=EXP2_REL_ERR) -> torch.Tensor:
    """Per row (float64): the sum of the e4m3 steps, as 2^(log2(step) + m) (m: the running max P was
    taken against, so that 2^(. - M) is the step relative to a final max M), of the P that lie within
    `rel_err` (relative; a scalar or per element) of a midpoint between two e4m3 values."""
    mant, ex = torch.frexp(p)                                    # p = mant * 2^ex, mant in [0.5, 1)
    step_units = mant * 16.0                                     # p in units of the e4m3 step 2^(ex - 4)
    dist = (step_units - step_units.floor() - 0.5).abs() / step_units
    near = (p > 0) & (dist < rel_err)
    lg = (ex - 4).double() + m.double()[:, None]
    return torch.where(near, torch.exp2(lg), torch.zeros_like(lg)).sum(dim=1)


def _attn_tile(qf, qs, kf, vf, ks, t0, t1, pv_accum, sm_log2, state, tail, amb=None):
    """One 64-key tile [t0, t1) of the kernel loop (one K scale `ks`), continuing from `state`
    (running max m, row sum d, unnormalized O) when given: returns the updated (m, d, O)."""
    r, d = qf.shape[0], vf.shape[1]
    if state is None:
        m = torch.full((r,), -math.inf)
        dsum = torch.zeros(r)
        acc = torch.zeros(r, d)
    else:
        m, dsum, acc = state
    s_int = qf @ kf[t0:t1].T                                     # exact integers (|S| < 2^21)
    dq = (qs * ks).float()                                        # fl(q_s * k_s) per row
    neg_off = torch.tensor(-S_FP8_OFFSET, dtype=torch.float32)
    if tail:
        rs = (s_int.double() * dq.double()[:, None]).float()     # fl(S * dequant)
        scale = sm_log2.expand(r)
    else:
        rs = s_int
        scale = (sm_log2 * dq).float()                            # fl(sm * dequant)
    m_t = _fma32(rs.max(dim=1).values, scale, neg_off.expand(r))
    m_new = torch.maximum(m, m_t)
    alpha = torch.exp2(m - m_new)
    x = _fma32(rs, scale[:, None], -m_new[:, None])
    p = torch.exp2(x)
    dsum = dsum * alpha + p.sum(dim=1)
    if amb is not None:
        rel = EXP2_REL_ERR if tail else bulk_rel_err(x, scale, m_new)
        amb += _ambiguous_steps(p, m_new, rel)
    pq = e4m3_to_float(e4m3_rn_satfinite(p))
    if pv_accum == "fp16":
        tile_acc = torch.zeros(r, d)
        for c0 in range(0, t1 - t0, 32):                         # m16n8k32 steps
            c1 = min(c0 + 32, t1 - t0)
            tile_acc = (tile_acc + pq[:, c0:c1] @ vf[t0 + c0:t0 + c1]).half().float()
    else:
        tile_acc = pq @ vf[t0:t1]
    acc = acc * alpha[:, None] + tile_acc
    return m_new, dsum, acc


def sage_attention(q, k, v, sm_scale=None, **kw):
    """`sageattn(q, k, v, tensor_layout="NHD", is_causal=False, sm_scale)` (attention.py:34),
    emulated on the CPU: quantize, then the kernel emulation. Returns bf16 [B, Lq, H, D]."""
    qq = quantize_qkv(q, k, v)
    o = attn_from_codes(qq["q_codes"], qq["q_scale"], qq["k_codes"], qq["k_scale"],
                        qq["v_codes"], qq["v_scale"], sm_scale=sm_scale, **kw)
    return o.to(q.dtype)


def sdpa_fp32(q, k, v, sm_scale=None, rows=None, heads=None):
    """Unquantized fp32 attention, the accuracy baseline reported beside every comparison."""
    b, lq, h, d = q.shape
    if sm_scale is None:
        sm_scale = d ** -0.5
    rows = torch.arange(lq) if rows is None else torch.as_tensor(rows)
    heads = list(range(h)) if heads is None else list(heads)
    out = torch.zeros(b, lq, h, d, dtype=torch.float32)
    for bi in range(b):
        for hi in heads:
            s = (q[bi, rows, hi].float() @ k[bi, :, hi].float().T) * sm_scale
            out[bi, rows, hi] = torch.softmax(s, dim=-1) @ v[bi, :, hi].float()
    return out


def compare(a: torch.Tensor, b: torch.Tensor, exclude: torch.Tensor | None = None) -> dict:
    """Error metrics used throughout (splitkv/check.py:48-56). `exclude` ([B, Lq, H] bool, the
    `ambiguous` rows of attn_from_codes) drops those rows from max_abs only; `excluded` counts them."""
    keep = None if exclude is None else (~exclude)[..., None].expand_as(a).flatten()
    a, b = a.double().flatten(), b.double().flatten()
    dlt = (a - b).abs()
    return dict(cos=F.cosine_similarity(a, b, dim=0).item(),
                max_abs=(dlt if keep is None else dlt[keep]).max().item(),
                rel_l2=((a - b).norm() / b.norm()).item(),
                excluded=0 if exclude is None else int(exclude.sum()))
