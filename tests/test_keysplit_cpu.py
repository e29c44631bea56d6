"""Key-range sequence split (lingbot_b200.split.KeySplitAttention), without a GPU: the memory tiles are
dealt out once each, the merge of per-rank key-range partials (fp16 O / row sum with (max, sum), the
form the attention kernel sends) reproduces the whole-window result in the CPU emulation, and the new C
ABI entry points reject bad arguments before any CUDA call."""
import ctypes

import pytest
import torch

from lingbot_b200 import _lib, split
from oracle import sage_semantics as O


@pytest.mark.parametrize("mem", [64, 640, 24128, 48256])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_key_tiles_cover_the_memory_once(mem, world):
    tiles = -(-mem // 128)
    got = [split.key_tiles(mem, world, r) for r in range(world)]
    assert got[0][0] == 0 and got[-1][1] == tiles
    for (a0, a1), (b0, b1) in zip(got, got[1:]):
        assert a1 == b0
    sizes = [t1 - t0 for t0, t1 in got]
    assert max(sizes) - min(sizes) <= 1


def _rank_ranges(mem, n, world, rank):
    """Key ranges (window coordinates) rank `rank` attends: its memory tiles and its chunk share."""
    part = split.share_part(n, world)
    t0, t1 = split.key_tiles(mem, world, rank) if mem else (0, 0)
    lo = min(n, rank * part)
    hi = min(n, lo + part)
    return [(t0 * 128, min(mem, t1 * 128)), (mem + lo, mem + hi)]


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("mem,n", [(640, 300), (576, 257), (0, 700)])
def test_key_range_merge_matches_whole_window(world, mem, n):
    """Merging every rank's key-range partials sent as fp16 O / row sum equals the same key ranges merged
    in fp32 up to fp16 rounding, stays within the Sage tolerance of the whole window (the P grid
    follows each range's running max, as with split-KV), and is as close to fp32 attention as the
    whole-window result (fp32 P.V, as the kernel)."""
    g = torch.Generator().manual_seed(5 + world)
    lq, h = 160, 2
    q = torch.randn(1, lq, h, 128, generator=g).bfloat16()
    k = (torch.randn(1, mem + n, h, 128, generator=g) + 2 * torch.randn(1, 1, h, 128, generator=g)).bfloat16()
    v = torch.randn(1, mem + n, h, 128, generator=g).bfloat16()
    qq = O.quantize_qkv(q, k, v)
    codes = (qq["q_codes"], qq["q_scale"], qq["k_codes"], qq["k_scale"], qq["v_codes"], qq["v_scale"])
    kernel = dict(pv_accum="fp32")
    ranges = [_rank_ranges(mem, n, world, rank) for rank in range(world)]     # one partial per rank
    covered = sorted(r for pieces in ranges for r in pieces if r[1] > r[0])
    assert covered[0][0] == 0 and covered[-1][1] == mem + n
    assert all(a[1] == b[0] for a, b in zip(covered, covered[1:]))     # every key exactly once
    merged = O.attn_from_codes(*codes, **kernel, key_ranges=ranges, partial_fp16=True)
    # measured: cos > 0.99999997, max-abs < 1e-4
    exact = O.compare(merged, O.attn_from_codes(*codes, **kernel, key_ranges=ranges))
    assert exact["cos"] >= 0.9999999 and exact["max_abs"] <= 2e-4, exact
    sage = O.compare(merged, O.attn_from_codes(*codes))
    assert sage["cos"] >= 0.9995 and sage["max_abs"] <= 2e-2, sage
    f32 = O.sdpa_fp32(q, k, v)
    whole = O.attn_from_codes(*codes, **kernel)
    assert O.compare(merged, f32)["cos"] >= O.compare(whole, f32)["cos"] - 1e-4


def _err():
    return _lib._lib.lbq_last_error()


def test_key_split_entry_points_check_their_arguments():
    lib = _lib.load()
    fake = ctypes.c_void_p(0x10000)          # never dereferenced: the checks fail first
    act = (fake, 1536, 1536, 128)
    # tile-range quantizer: the range must hold valid tokens and map to source tokens >= 0
    args = (*act, *act, 1, 12, -256, 1, 2, 640, 640, 1280, fake, fake, fake, fake, fake, fake, fake, 0)
    assert lib.lbq_quant_kv_tiles(*args, 1, 3, None) == 1 and b"source token" in _err()
    assert lib.lbq_quant_kv_tiles(*args, 2, 7, None) == 1 and b"tiles [2, 7)" in _err()
    # key-range attention
    lt0, tiles, valid = (ctypes.c_int * 2)(0, 2), (ctypes.c_int * 2)(5, 3), (ctypes.c_int * 2)(640, 300)
    base = (fake, fake, 300, 384, fake, fake, fake, 2, 640, 1, 2, 0.0)
    tail = (fake, 2, 0, 0, 256, 0, 1 << 20, None)
    assert lib.lbq_attn_fwd_keys(*base, lt0, tiles, valid, *tail) == 1 and b"range 1" in _err()
    tiles[1] = 1
    assert lib.lbq_attn_fwd_keys(*base, lt0, tiles, valid, fake, 2, 0, 0, 100, 0, 1 << 20, None) == 1
    assert b"part 100" in _err()
    assert lib.lbq_attn_fwd_keys(*base, lt0, tiles, valid, fake, 2, 2, 0, 256, 0, 1 << 20, None) == 1
    assert b"rank 2" in _err()
    zero = (ctypes.c_int * 2)(0, 0)
    assert lib.lbq_attn_fwd_keys(*base, lt0, zero, valid, *tail) == 1 and b"empty key range" in _err()
    # combine and query push
    assert lib.lbq_keys_combine(fake, fake, 2, 256, 300, fake, 1, 2, *act, None) == 1 and b"rows 300" in _err()
    assert lib.lbq_q_push(fake, fake, 128, 64, 512, 1, 2, 0, 0, fake, 2, 0, 0, 0, None) == 1
    assert b"multiples of 128" in _err()


def test_key_ranges_restate_the_split_emulation():
    """The oracle's key-range partials are the split-KV partials generalised: one whole-window range is
    the unsplit emulation, and the split ranges as key ranges are `splits` exactly."""
    g = torch.Generator().manual_seed(2)
    q = torch.randn(1, 96, 2, 128, generator=g).bfloat16()
    k = torch.randn(1, 700, 2, 128, generator=g).bfloat16()
    v = torch.randn(1, 700, 2, 128, generator=g).bfloat16()
    qq = O.quantize_qkv(q, k, v)
    codes = (qq["q_codes"], qq["q_scale"], qq["k_codes"], qq["k_scale"], qq["v_codes"], qq["v_scale"])
    kernel = dict(pv_accum="fp32")
    assert torch.equal(O.attn_from_codes(*codes, **kernel, key_ranges=[[(0, 700)]]),
                       O.attn_from_codes(*codes, **kernel))
    per = 2 * 128                                  # 6 tiles in 3 splits
    ranges = [[(s, min(700, s + per))] for s in range(0, 700, per)]
    assert torch.equal(O.attn_from_codes(*codes, **kernel, key_ranges=ranges),
                       O.attn_from_codes(*codes, **kernel, splits=3))
    # a partial made of two pieces runs them under one running max: the same as one piece
    assert torch.equal(O.attn_from_codes(*codes, **kernel, key_ranges=[[(0, 256), (256, 700)]]),
                       O.attn_from_codes(*codes, **kernel))


@pytest.mark.parametrize("mem,n", [(24128, 6032), (48256, 6032), (1280, 700), (0, 6032)])
@pytest.mark.parametrize("world", range(1, 9))
def test_every_rank_passes_the_abi_checks(mem, n, world):
    """The arguments KeySplitAttention gives lbq_attn_fwd_keys and lbq_quant_kv_tiles pass the ABI's
    validation for every rank (BASELINE config 4 and 5 windows among them): on a host without a GPU the
    calls then stop at the tensor map or the launch (LBQ_ERR_CUDA), never at an argument check."""
    if mem == 0 and n <= (world - 1) * split.share_part(n, world):
        pytest.skip("the last ranks hold no keys (KeySplitAttention rejects this split)")
    if mem and -(-mem // 128) < world:
        pytest.skip("fewer memory tiles than ranks (KeySplitAttention rejects this split)")
    lib = _lib.load()
    fake = ctypes.c_void_p(0x10000)
    part = split.share_part(n, world)
    nseg = 2 if mem else 1
    seg_len = mem if mem else n
    covered = 0
    for rank in range(world):
        rg = split.key_ranges(mem, n, world, rank)
        assert len(rg) == nseg and sum(t for _, t, _ in rg) >= 1
        arr = ctypes.c_int * nseg
        rc = lib.lbq_attn_fwd_keys(fake, fake, n, world * part, fake, fake, fake, nseg, seg_len, 1, 12, 0.0,
                                   arr(*[x[0] for x in rg]), arr(*[x[1] for x in rg]), arr(*[x[2] for x in rg]),
                                   fake, world, rank, 0, part, 1 << 20, 1 << 24, None)
        assert rc == 3, (rank, rc, _err())                              # LBQ_ERR_CUDA: validation passed
        act = (fake, 1536, 1536, 128)
        for s, (t0, nt, valid) in enumerate(rg):
            if nt == 0:
                continue
            chunk = s == nseg - 1
            lo = t0 * 128 if chunk else 0
            rc = lib.lbq_quant_kv_tiles(*act, *act, 1, 12, -lo if chunk else 0, s, nseg,
                                        (min(n, lo + part) if chunk else valid), seg_len, mem + n,
                                        fake, fake, fake, fake, fake, fake, fake, int(not chunk or mem == 0),
                                        t0, t0 + nt, None)
            assert rc == 3, (rank, s, rc, _err())
            covered += min(valid, (t0 + nt) * 128) - t0 * 128
    assert covered == mem + n                                            # every key of the window once
