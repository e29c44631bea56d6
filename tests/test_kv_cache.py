"""The KV-cache mirror against the reference's bookkeeping (lingbot/layers/kv_cache.py), replayed on the
golden write / rewrite / eviction schedule; and, on the GPU, the cache-aware attend (block statistics
kept by write/evict) against quantizing the same window from scratch — the check the reference runs in
experiments/bench_attn/sage_preq_check.py (bit identity of sage_preq.attend vs sageattn)."""
import pytest
import torch

from lingbot_b200 import kv_cache as kvc
from tests._golden import kv_schedule


def test_bookkeeping_matches_reference_schedule():
    sch = kv_schedule()
    torch.manual_seed(0)
    kc = kvc.allocate(1, [1, sch["T"], sch["H"], sch["D"]], torch.bfloat16, "cpu")[0]
    for st in sch["steps"]:
        n = st["n"]
        k = torch.randn(1, n, sch["H"], sch["D"]).bfloat16()
        v = torch.randn(1, n, sch["H"], sch["D"]).bfloat16()
        assert list(kvc.plan(kc, n, st["current_start"], sch["sink"], sch["local"])) == st["plan"]
        end, cur_end = kvc.write(kc, k, v, st["current_start"], sch["sink"], sch["local"])
        assert (end, cur_end) == (st["end"], st["current_end"])
        kw, _ = kvc.window(kc, end, sch["T"])
        assert [kw.shape[1]] == st["window"]
        assert float(kc["k"].double().sum()) == st["k_checksum"]
        assert float(kc["v"].double().sum()) == st["v_checksum"]
        kvc.commit(kc, cur_end, end)


@pytest.mark.gpu
def test_cache_attend_bit_identical_to_fresh_quantization():
    from lingbot_b200 import ops
    torch.manual_seed(0)
    dev, H, D = "cuda", 10, 128
    T, n_tok, sink, local = 1000, 300, 200, 10      # odd sizes on purpose (sage_preq_check.py:11-12)
    kc = kvc.allocate(1, [1, T, H, D], torch.bfloat16, dev)[0]

    def rnd(n):
        x = torch.randn(1, n, H, D, device=dev, dtype=torch.bfloat16)
        return x * (1 + 20 * (torch.rand(1, 1, H, D, device=dev) > 0.98))      # outlier channels

    start = 0
    for chunk in range(6):
        for rewrite in range(3):
            n = n_tok - (7 if chunk == 2 else 0)
            k, v, q = rnd(n), rnd(n), rnd(n)
            end, cur_end = kvc.write(kc, k, v, start, sink, local)
            out = kvc.attend(q, kc, end - n, end)
            ref = ops.sage_attn(q, kc["k"][:, :end], kc["v"][:, :end])
            torch.cuda.synchronize()
            assert torch.equal(out, ref), f"chunk {chunk} rewrite {rewrite} end {end}"
            kvc.commit(kc, cur_end, end)
        start += n
