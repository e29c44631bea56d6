"""Full-size parity through the bench's own path: the chunk's K/V written into a layer cache behind
its memory part (block statistics refreshed), the window re-quantized from the cached statistics, Q
quantized, attention, all captured in one CUDA graph and replayed as bench.py does. BASELINE config 4
(q 6032 x kv 30160: 24128 memory + 6032 chunk tokens) and config 5 (kv 54288: 48256 + 6032, K
channels 0-3 x20); the oracle checks 3 heads x 384 rows of the replayed output against the GPU's own
codes (the model of experiments/bench_attn/sage_preq_check.py:13-36), beside fp32 SDPA."""
import pytest
import torch

from oracle import sage_semantics as O
from tests.test_attn_gpu import check_parity

pytestmark = pytest.mark.gpu

H, D, LQ = 12, 128, 6032
ROWS = torch.cat([torch.arange(0, 128), torch.arange(2944, 3072), torch.arange(5904, 6032)])
HEADS = [0, 5, 11]


def _window_call(mem, outlier, seed):
    from lingbot_b200 import _lib, kv_cache, ops
    dev = torch.device("cuda")
    lk = mem + LQ
    g = torch.Generator(device=dev).manual_seed(seed)
    cache = kv_cache.allocate(1, [1, lk, H, D], torch.bfloat16, dev)[0]
    koff = torch.randn(1, 1, H, D, generator=g, device=dev) * 3.0
    cache["k"][:, :mem].normal_(generator=g).add_(koff)
    cache["v"][:, :mem].normal_(generator=g)
    if outlier:
        cache["k"][:, :mem, :, :4] *= 20.0
    kv_cache.refresh_stats(cache, 0, mem)
    q = torch.randn(1, LQ, H, D, generator=g, device=dev).bfloat16()
    kc = torch.randn(1, LQ, H, D, generator=g, device=dev) + koff
    if outlier:
        kc[..., :4] *= 20.0
    kc = kc.bfloat16()
    vc = torch.randn(1, LQ, H, D, generator=g, device=dev).bfloat16()
    quantizer = kv_cache.WindowQuantizer()
    out = torch.empty(1, LQ, H, D, dtype=torch.bfloat16, device=dev)
    box = {}

    def call():
        cache["k"][:, mem:lk] = kc
        cache["v"][:, mem:lk] = vc
        kv_cache.refresh_stats(cache, mem, lk)
        box["w"] = kv_cache.quantize_window(q, cache, lk, quantizer)
        ops.attn_from_codes(box["w"], out=out)

    call()                                   # warm-up (sizes the quantizer buffers)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    out.zero_()
    for _ in range(2):
        graph.replay()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return q, cache["k"][:, :lk], cache["v"][:, :lk], box["w"], out


@pytest.mark.parametrize("cfg", ["config4", "config5"])
def test_full_size_window_through_the_bench_path(cfg):
    mem, outlier = (24128, False) if cfg == "config4" else (48256, True)
    q, k, v, w, out = _window_call(mem, outlier, seed=1234 if cfg == "config4" else 5000)
    got = out.float().cpu()
    exact, sage = check_parity(got, w, rows=ROWS, heads=HEADS)
    fp32 = O.sdpa_fp32(q.cpu(), k.cpu(), v.cpu(), rows=ROWS, heads=HEADS)[:, ROWS][:, :, HEADS]
    m32 = O.compare(got[:, ROWS][:, :, HEADS], fp32)
    # Sage's own accuracy on randn at the production shape is cos 0.99925 against fp32 (the
    # reference's record, results/h2_cfg_base.json); the outlier channels cost more
    assert m32["cos"] >= (0.999 if cfg == "config4" else 0.99), m32
