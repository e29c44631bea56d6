"""Generate the golden fixtures in this directory from the reference's OWN code.

Run where the reference is checked out (--ref or LINGBOT_REF). The GPU box never runs this: it only
reads the committed .npz / .json outputs.

    python tests/golden/make_golden.py --ref <path to lingbot-world-v2-realtime>

What it records:
  * quant_*.npz — inputs (bf16 bits) and the outputs of the reference's torch quantizers
    `experiments/modules/sage_kvq.py` `_quant_int8` (Q: 32-token groups padded to 128; K: 64-token
    blocks after subtracting km = k.mean over the window) and `_quant_v_fp8` (V: per-channel e4m3 in
    Sage's permuted [B, D, H, n] layout, amax = max |v| over the window, no margin), exactly as
    `lingbot/layers/sage_preq.py:115-124` drives Sage's quantizers per call.
  * rope_grid2x4x6.npz — the reference's RoPE: its `rope_params` table
    (reference/wan/modules/model.py:29-36) as the DiT builds it (lingbot/models/lingbot_world/
    transformer.py:553-558), `causal_rope_freqs` for a two-sample batch (transformer.py:53-76) and
    `causal_rope_apply` of a bf16 input (transformer.py:134-146). transformer.py itself imports
    diffusers and the Wan model, so the three functions are taken from its source text and run alone.
  * fp8_linear.npz — the reference's rowwise FP8Linear (lingbot/layers/linear.py:10-31) built from a
    seeded bf16 nn.Linear: its e4m3 weights and row scales, and the e4m3 activations and row scales
    its forward hands to torch._scaled_mm (recorded by intercepting that call, which has no rowwise CPU
    kernel), for an input with a zero row.
  * kv_schedule.json — the host bookkeeping of `lingbot/layers/kv_cache.py` (plan/evict/write/
    window/commit) over the write / rewrite / eviction schedule of
    `experiments/bench_attn/sage_preq_check.py:11-36`, with float64 (order-independent) checksums of the cache buffers after
    every write.
"""
import argparse
import importlib.util
import json
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def load_functions(path, names, env):
    """The named top-level functions of a source file, compiled on their own into `env`."""
    import ast
    src = open(path).read()
    tree = ast.parse(src)
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in names:
            exec(compile(ast.Module(body=[node], type_ignores=[]), path, "exec"), env)
    missing = [n for n in names if n not in env]
    assert not missing, missing
    return env


def rope_golden(ref):
    env = {"torch": torch, "_ROPE_FP32C": False}
    load_functions(os.path.join(ref, "reference/wan/modules/model.py"), ["rope_params"], env)
    load_functions(os.path.join(ref, "lingbot/models/lingbot_world/transformer.py"),
                   ["causal_rope_freqs", "causal_rope_apply"], env)
    d = 128
    freqs = torch.view_as_real(torch.cat([env["rope_params"](1024, d - 4 * (d // 6)),
                                          env["rope_params"](1024, 2 * (d // 6)),
                                          env["rope_params"](1024, 2 * (d // 6))], dim=1))
    grid = [(2, 4, 6), (2, 4, 6)]
    cos, sin = env["causal_rope_freqs"](grid, freqs, start_frame=5)          # [B, L, 1, 64] each
    g = torch.Generator().manual_seed(77)
    x = (torch.randn(2, 48, 2, d, generator=g) * 2.0).bfloat16()
    out = env["causal_rope_apply"](x, (cos, sin))
    # the first 16 positions of the table cover every frame, row and column used here
    return dict(freqs16=freqs[:16].numpy(), grid=np.array(grid), start_frame=np.array(5),
                cos=cos[:, :, 0].numpy(), sin=sin[:, :, 0].numpy(), x=bf16_bits(x), out=bf16_bits(out))


def fp8_golden(ref):
    lin_mod = load(os.path.join(ref, "lingbot/layers/linear.py"), "ref_linear")
    g = torch.Generator().manual_seed(88)
    lin = torch.nn.Linear(256, 96).bfloat16()
    with torch.no_grad():
        lin.weight.copy_((torch.randn(96, 256, generator=g) * 0.05).bfloat16())
        lin.bias.copy_((torch.randn(96, generator=g) * 0.1).bfloat16())
    f = lin_mod.FP8Linear(lin)
    x = (torch.randn(7, 256, generator=g) * 3).bfloat16()
    x[3] = 0
    seen = {}

    def record(a, b, scale_a=None, scale_b=None, bias=None, out_dtype=None):
        seen.update(x8=a, xs=scale_a, w8t=b, ws=scale_b)
        return torch.zeros(a.shape[0], b.shape[1], dtype=out_dtype)
    real = torch._scaled_mm
    torch._scaled_mm = record
    try:
        f(x)
    finally:
        torch._scaled_mm = real
    u8 = lambda t: t.contiguous().view(torch.uint8).numpy()  # noqa: E731
    return dict(weight=bf16_bits(lin.weight.detach()), bias=bf16_bits(lin.bias.detach()), x=bf16_bits(x),
                w8=u8(f.w8), w_scale=f.w_scale_t.numpy(), x8=u8(seen["x8"]), x_scale=seen["xs"].numpy(),
                w8_seen=u8(seen["w8t"].t()), w_scale_seen=seen["ws"].numpy())


def bf16_bits(x):
    return x.contiguous().view(torch.int16).numpy()


# (name, heads, q_len, kv_len, k_offset_std, outlier) — odd lengths from splitkv/check.py:58-63,
# outlier channels from sage_preq_check.py:20-22 and BASELINE config 5 (4 of 128 channels x20).
CASES = [
    ("base_q300_kv1000", 2, 300, 1000, 3.0, None),
    ("kv65_q300", 2, 300, 65, 3.0, None),
    ("kv64_q128", 1, 128, 64, 3.0, None),
    ("kv4097_q513", 1, 513, 4097, 3.0, None),
    ("outlier_rand_q257_kv777", 2, 257, 777, 3.0, "rand"),
    ("outlier4of128_q96_kv2048", 2, 96, 2048, 3.0, "four"),
    ("q1_kv1", 1, 1, 1, 0.0, None),
]


def make_inputs(seed, h, nq, nk, koff, outlier):
    g = torch.Generator().manual_seed(seed)
    d = 128
    q = torch.randn(1, nq, h, d, generator=g)
    k = torch.randn(1, nk, h, d, generator=g)
    v = torch.randn(1, nk, h, d, generator=g)
    if koff:
        k = k + torch.randn(1, 1, h, d, generator=g) * koff
    if outlier == "rand":
        mask = (torch.rand(1, 1, h, d, generator=g) > 0.98).float()
        k = k * (1 + 20 * mask)
        v = v * (1 + 20 * mask)
    elif outlier == "four":
        k[..., :4] *= 20
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def quant_case(kvq, seed, h, nq, nk, koff, outlier):
    q, k, v = make_inputs(seed, h, nq, nk, koff, outlier)
    q_codes, q_scale = kvq._quant_int8(q, kvq.WARP_Q, kvq.BLK_Q)
    km = k.mean(dim=1, keepdim=True)
    k_codes, k_scale = kvq._quant_int8(k, kvq.BLK_K, kvq.BLK_K, km)
    v_amax = v.abs().amax(dim=1).float()
    e16 = (nk + 15) // 16 * 16
    vp = torch.nn.functional.pad(v, (0, 0, 0, 0, 0, e16 - nk))
    v_sage = kvq._quant_v_fp8(vp, v_amax)                      # [B, D, H, e16] permuted
    return dict(q=bf16_bits(q), k=bf16_bits(k), v=bf16_bits(v),
                q_codes=q_codes.numpy(), q_scale=q_scale.numpy(),
                km=bf16_bits(km), k_codes=k_codes.numpy(), k_scale=k_scale.numpy(),
                v_amax=v_amax.numpy(), v_scale=(v_amax / kvq.V_SCALE_MAX).numpy(),
                v_codes_sage=v_sage.contiguous().view(torch.uint8).numpy())


def kv_schedule(kvc):
    """sage_preq_check.py:11-36: window T=1000, 300-token chunks (one of 293), sink 200,
    6 chunks x 3 rewrites. The check script starts chunk c at c*300 even after the 293-token
    chunk, which overflows the 1000-token buffer on chunk 3 (kv_cache.write raises a shape
    error); here chunk starts are the running token count, as the pipeline passes them."""
    torch.manual_seed(0)
    H, D = 2, 128
    T, n_tok, sink, local = 1000, 300, 200, 10
    kc = kvc.allocate(1, [1, T, H, D], torch.bfloat16, "cpu")[0]
    steps = []
    start = 0
    for chunk in range(6):
        for rewrite in range(3):
            n = n_tok - (7 if chunk == 2 else 0)
            k = torch.randn(1, n, H, D).bfloat16()
            v = torch.randn(1, n, H, D).bfloat16()
            plan = kvc.plan(kc, n, start, sink, local)
            end, cur_end = kvc.write(kc, k, v, start, sink, local)
            kw, vw = kvc.window(kc, end, T)
            steps.append(dict(chunk=chunk, rewrite=rewrite, n=n, current_start=start,
                              plan=list(plan), end=end, current_end=cur_end,
                              window=[int(kw.shape[1])],
                              k_checksum=float(kc["k"].double().sum()),
                              v_checksum=float(kc["v"].double().sum())))
            kvc.commit(kc, cur_end, end)
        start += n
    return dict(T=T, n_tok=n_tok, sink=sink, local=local, H=H, D=D, steps=steps)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("LINGBOT_REF"),
                    help="checkout of the reference project (or set LINGBOT_REF)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference checkout with --ref or LINGBOT_REF")
    kvq = load(os.path.join(args.ref, "experiments/modules/sage_kvq.py"), "ref_sage_kvq")
    kvc = load(os.path.join(args.ref, "lingbot/layers/kv_cache.py"), "ref_kv_cache")
    torch.set_num_threads(4)
    for i, (name, h, nq, nk, koff, outlier) in enumerate(CASES):
        out = quant_case(kvq, 1000 + i, h, nq, nk, koff, outlier)
        meta = np.array(json.dumps(dict(name=name, heads=h, q_len=nq, kv_len=nk, seed=1000 + i,
                                        k_offset_std=koff, outlier=outlier)))
        np.savez_compressed(os.path.join(HERE, f"quant_{name}.npz"), meta=meta, **out)
        print("wrote", name)
    np.savez_compressed(os.path.join(HERE, "rope_grid2x4x6.npz"), **rope_golden(args.ref))
    np.savez_compressed(os.path.join(HERE, "fp8_linear.npz"), **fp8_golden(args.ref))
    print("wrote fp8_linear.npz")
    print("wrote rope_grid2x4x6.npz")
    with open(os.path.join(HERE, "kv_schedule.json"), "w") as f:
        json.dump(kv_schedule(kvc), f, indent=1)
    print("wrote kv_schedule.json")


if __name__ == "__main__":
    main()
