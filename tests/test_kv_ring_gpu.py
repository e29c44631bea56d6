"""Eviction as an index remap (kv_cache.allocate(..., ring=True)) against the reference's left-shift
eviction (lingbot/layers/kv_cache.py:52-61, mirrored by the default cache): over a write / rewrite /
eviction schedule, the ring cache must give the same quantized window (codes, scales, km), the same
attention output bits, the same logical window and the same block statistics, while its eviction moves
no K/V rows."""
import pytest
import torch

from lingbot_b200 import kv_cache as kvc

pytestmark = pytest.mark.gpu


def _rnd(g, n, h, dev):
    x = torch.randn(1, n, h, 128, generator=g, device=dev)
    return (x * (1 + 20 * (torch.rand(1, 1, h, 128, generator=g, device=dev) > 0.98))).bfloat16()


def _nblocks(end):
    return (end + 63) // 64


@pytest.mark.parametrize("T,n_tok,sink,short", [(1000, 300, 200, 7), (1024, 256, 128, 0)],
                         ids=["golden_schedule_unaligned", "aligned_64"])
def test_ring_cache_matches_the_shifting_cache(T, n_tok, sink, short):
    """T / chunk / sink of the reference's check (experiments/bench_attn/sage_preq_check.py:11-36:
    window 1000, 300-token chunks with one of 293, sink 200, three rewrites per chunk), and a
    64-aligned variant where evictions move statistics rows instead of recomputing them."""
    dev, H, local = "cuda", 4, 10
    g = torch.Generator(device=dev).manual_seed(3)
    shift = kvc.allocate(1, [1, T, H, 128], torch.bfloat16, dev)[0]
    ring = kvc.allocate(1, [1, T, H, 128], torch.bfloat16, dev, ring=True)[0]
    start, evictions, moved_head = 0, 0, False
    for chunk in range(7):
        for rewrite in range(3):
            n = n_tok - (short if chunk == 2 else 0)
            k, v, q = _rnd(g, n, H, dev), _rnd(g, n, H, dev), _rnd(g, n, H, dev)
            evicted = kvc.plan(shift, n, start, sink, local)[0]
            evictions += evicted > 0
            outs, wins = [], []
            for c in (shift, ring):
                end, cur_end = kvc.write(c, k, v, start, sink, local)
                w = kvc.quantize_window(q, c, end, kvc.WindowQuantizer())
                wins.append((w, end))
                outs.append(kvc.attend(q, c, end - n, end, quantizer=kvc.WindowQuantizer()).clone())
                kvc.commit(c, cur_end, end)
            torch.cuda.synchronize()
            (w0, e0), (w1, e1) = wins
            assert e0 == e1
            for name in ("q_codes", "q_scale", "k_codes", "k_scale", "vt_codes", "v_scale", "km"):
                a, b = getattr(w0, name), getattr(w1, name)
                assert torch.equal(a.view(torch.uint8), b.view(torch.uint8)), (chunk, rewrite, name)
            assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16)), (chunk, rewrite)
            k0, v0 = kvc.window(shift, e0, T)
            k1, v1 = kvc.window(ring, e1, T)
            assert torch.equal(k0.view(torch.int16), k1.view(torch.int16))
            assert torch.equal(v0.view(torch.int16), v1.view(torch.int16))
            nb = _nblocks(e0)
            assert torch.equal(shift["lbq_ksum"][:, :nb].view(torch.int64), ring["lbq_ksum"][:, :nb].view(torch.int64))
            assert torch.equal(shift["lbq_vamax"][:, :nb].view(torch.int32), ring["lbq_vamax"][:, :nb].view(torch.int32))
            moved_head |= ring["lbq_ring_head"] != 0
        start += n
    assert evictions > 0 and moved_head          # the schedule did evict, and the ring did rotate
