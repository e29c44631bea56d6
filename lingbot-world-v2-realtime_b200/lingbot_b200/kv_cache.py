"""Self-attention KV cache of the causal DiT — drop-in for lingbot/layers/kv_cache.py — plus the
quantized attention over its window that replaces lingbot/layers/sage_preq.py:attend.

The bookkeeping (`plan`, `evict`, `write`, `window`, `commit`) has the reference's semantics and
host-int indices (kv_cache.py:11-88). What is new is a table of per-64-token-block statistics kept
beside each layer's K/V (fp64 K sums and max |V| per channel, the generalisation of sage_preq's
V min/max table, sage_preq.py:36-44,87-104): `write` refreshes the blocks it touched and `evict`
the blocks after the sink, so `attend` re-quantizes the window with one read of the bf16 cache
(window sums -> K/V codes) instead of two.

With `allocate(..., ring=True)` the part of the buffer after the sink is a ring: an eviction moves
a head index instead of shifting the window left by a copy (the reference's kv_cache.py:52-61; its
ring-buffer attempt is experiments/modules/model_fast_kv_ring.py). Logical window token t — the row
the reference would hold it in — lives at row t below the sink, else at
sink + ((t - sink + head) mod (size - sink)); the cache kernels read and write through that map, and
the quantized codes come out in logical order, so the attention is the same call. The statistics
are kept per logical block: when the sink and the eviction are multiples of 64 tokens an eviction
moves the rows of the table (a few MB) and nothing is re-read; otherwise the blocks after the sink
are recomputed through the map (one read, where the shift costs a read and a write more). `window`
of a ring cache materialises the logical slice (a copy), for callers that need bf16 K/V.
"""
from __future__ import annotations

import torch

from . import _lib, ops

BLK = 64


def _stats_tables(shape, device):
    b, kv_size, h, d = shape
    nb = (kv_size + BLK - 1) // BLK
    return (torch.zeros(b, nb, h, d, dtype=torch.float64, device=device),
            torch.zeros(b, nb, h, d, dtype=torch.float32, device=device))


def heap_bytes(num_layers, shape, dtype):
    """Peer-heap bytes that `allocate(num_layers, shape, dtype, device, heap)` carves (K, V and the
    block tables of every layer, each at a 256-byte aligned offset)."""
    b, kv_size, h, d = shape
    nb = (kv_size + BLK - 1) // BLK
    esz = torch.empty((), dtype=dtype).element_size()
    up = lambda x: (x + 255) // 256 * 256  # noqa: E731
    return num_layers * (2 * up(b * kv_size * h * d * esz) + up(b * nb * h * d * 8) + up(b * nb * h * d * 4))


def allocate(num_layers, shape, dtype, device, heap=None, ring=False):
    """One cache dict per layer; `shape` is [batch, window tokens, heads, head_dim] (kv_cache.py:11-20).
    With a `peer.PeerHeap`, K, V and the block tables are carved from it (zeroed) so that the other
    ranks of a sequence split can write the current chunk straight into this rank's replica.
    ring=True: evictions move a ring head instead of copying (GPU caches; not with a peer heap)."""
    if ring and heap is not None:
        raise ValueError("a ring cache is per GPU: the sequence split's peer pushes write logical rows")
    caches = []
    for _ in range(num_layers):
        if heap is None:
            ksum, vamax = _stats_tables(shape, device)
            k = torch.zeros(shape, dtype=dtype, device=device)
            v = torch.zeros(shape, dtype=dtype, device=device)
        else:
            b, kv_size, h, d = shape
            nb = (kv_size + BLK - 1) // BLK
            k, v = heap.carve(shape, dtype), heap.carve(shape, dtype)
            ksum, vamax = heap.carve((b, nb, h, d), torch.float64), heap.carve((b, nb, h, d), torch.float32)
        caches.append({
            'k': k,
            'v': v,
            'global_end_index': torch.tensor([0], dtype=torch.long, device=device),
            'local_end_index': torch.tensor([0], dtype=torch.long, device=device),
            'global_end_int': 0,
            'local_end_int': 0,
            'lbq_ksum': ksum,
            'lbq_vamax': vamax,
            'lbq_ring': bool(ring),
            'lbq_ring_sink': None,
            'lbq_ring_head': 0,
        })
    return caches


def ring_args(kv_cache):
    """(sink, len, head) of a ring cache for the C ABI; (0, 0, 0) otherwise or before its first eviction
    fixed the sink."""
    sink = kv_cache.get("lbq_ring_sink")
    if not kv_cache.get("lbq_ring") or sink is None:
        return 0, 0, 0
    return sink, kv_cache["k"].shape[1] - sink, kv_cache["lbq_ring_head"]


def _ring_sink(kv_cache, sink_tokens):
    """Fix (first call) or check the sink size of a ring cache."""
    if not kv_cache.get("lbq_ring"):
        return
    if kv_cache["lbq_ring_sink"] is None:
        if not kv_cache["k"].is_cuda:
            raise ValueError("ring caches are GPU caches")
        kv_cache["lbq_ring_sink"] = int(sink_tokens)
    elif kv_cache["lbq_ring_sink"] != sink_tokens:
        raise ValueError(f"ring cache built for a {kv_cache['lbq_ring_sink']}-token sink, called with {sink_tokens}")


def plan(kv_cache, num_new_tokens, current_start, sink_tokens, local_attn_size):
    """Host-side bookkeeping of `write` (kv_cache.py:23-49):
    (evicted, rolled, local_start_index, local_end_index, current_end)."""
    current_end = current_start + num_new_tokens
    kv_cache_size = kv_cache["k"].shape[1]
    global_end = kv_cache.get("global_end_int")
    if global_end is None:
        global_end = kv_cache["global_end_index"].item()
        local_end = kv_cache["local_end_index"].item()
    else:
        local_end = kv_cache["local_end_int"]
    evicted = rolled = 0
    if local_attn_size == -1:
        local_end_index = current_end
        local_start_index = current_start
    elif (current_end > global_end) and (num_new_tokens + local_end > kv_cache_size):
        evicted = num_new_tokens + local_end - kv_cache_size
        rolled = local_end - evicted - sink_tokens
        local_end_index = local_end + current_end - evicted - global_end
        local_start_index = local_end_index - num_new_tokens
    else:
        local_end_index = local_end + current_end - global_end
        local_start_index = local_end_index - num_new_tokens
    return evicted, rolled, local_start_index, local_end_index, current_end


def refresh_stats(kv_cache, tok_begin, tok_end):
    """Recompute the block statistics of the blocks covering tokens [tok_begin, tok_end) of the
    buffer (tokens past tok_end inside the last block count as absent until written)."""
    k, v = kv_cache["k"], kv_cache["v"]
    if "lbq_ksum" not in kv_cache:
        kv_cache["lbq_ksum"], kv_cache["lbq_vamax"] = _stats_tables(tuple(k.shape), k.device)
    if tok_end <= tok_begin or not k.is_cuda:
        return
    b, kv_size, h, _ = k.shape
    ksum, vamax = kv_cache["lbq_ksum"], kv_cache["lbq_vamax"]
    _lib.call("lbq_kv_block_stats", ops._ptr(k), *k.stride()[:3], ops._ptr(v), *v.stride()[:3], b, h, tok_end,
              tok_begin // BLK, (tok_end + BLK - 1) // BLK, ksum.shape[1], ops._ptr(ksum), ops._ptr(vamax),
              *ring_args(kv_cache), ops._stream())


def evict(kv_cache, sink_tokens, evicted, rolled):
    """Drop the oldest `evicted` tokens after the sink, keeping the `rolled` after them
    (kv_cache.py:52-61): the reference shifts them left by a copy; a ring cache advances its head.
    Then the block statistics of the tokens after the sink are brought up to date."""
    _ring_sink(kv_cache, sink_tokens)
    if kv_cache.get("lbq_ring"):
        size = kv_cache["k"].shape[1]
        kv_cache["lbq_ring_head"] = (kv_cache["lbq_ring_head"] + evicted) % (size - sink_tokens)
        if sink_tokens % BLK == 0 and evicted % BLK == 0 and "lbq_ksum" in kv_cache:
            # logical block b now holds what block b + evicted/64 held: move the statistics rows
            b0, sh = sink_tokens // BLK, evicted // BLK
            nfull = rolled // BLK
            for t in (kv_cache["lbq_ksum"], kv_cache["lbq_vamax"]):
                t[:, b0:b0 + nfull] = t[:, b0 + sh:b0 + sh + nfull].clone()
            if rolled % BLK:                                   # the partial last block: recompute
                refresh_stats(kv_cache, sink_tokens + nfull * BLK, sink_tokens + rolled)
            return
        refresh_stats(kv_cache, sink_tokens, sink_tokens + rolled)
        return
    kv_cache["k"][:, sink_tokens:sink_tokens + rolled] = \
        kv_cache["k"][:, sink_tokens + evicted:sink_tokens + evicted + rolled].clone()
    kv_cache["v"][:, sink_tokens:sink_tokens + rolled] = \
        kv_cache["v"][:, sink_tokens + evicted:sink_tokens + evicted + rolled].clone()
    refresh_stats(kv_cache, sink_tokens, sink_tokens + rolled)


def _rope_args(rope):
    """(cos, sin) float64 tables [B, L, 64] (or the reference's [B, L, 1, 64]) -> C-ABI arguments."""
    if rope is None:
        return None, None, 0, 0
    cos, sin = rope
    if cos.dim() == 4:
        cos, sin = cos[:, :, 0], sin[:, :, 0]
    for t in (cos, sin):
        if t.dtype != torch.float64 or not t.is_cuda or t.stride(-1) != 1 or t.shape[-1] != 64:
            raise ValueError("rope tables must be CUDA float64 [B, L, 64] with unit last stride")
    if cos.stride() != sin.stride():
        raise ValueError("rope cos and sin tables must share strides")
    return ops._ptr(cos), ops._ptr(sin), cos.stride(0), cos.stride(1)


def store(kv_cache, k, v, tok_begin, rope=None):
    """Store K/V at tokens [tok_begin, tok_begin + n) of the cache buffers and refresh the statistics
    of the blocks they touch, in one kernel (lbq_cache_write); with `rope` = the chunk's (cos, sin)
    tables, K is roped on the way (the reference ropes it before kv_cache.write,
    transformer.py:213-219)."""
    kc, vc = kv_cache["k"], kv_cache["v"]
    if "lbq_ksum" not in kv_cache:
        kv_cache["lbq_ksum"], kv_cache["lbq_vamax"] = _stats_tables(tuple(kc.shape), kc.device)
    b, n, h, _ = k.shape
    ksum, vamax = kv_cache["lbq_ksum"], kv_cache["lbq_vamax"]
    rc, rs, sr_b, sr_l = _rope_args(rope)
    _lib.call("lbq_cache_write", ops._ptr(k), *k.stride()[:3], ops._ptr(v), *v.stride()[:3], rc, rs, sr_b, sr_l,
              ops._ptr(kc), *kc.stride()[:3], ops._ptr(vc), *vc.stride()[:3], b, h, kc.shape[1], tok_begin, n,
              ksum.shape[1], ops._ptr(ksum), ops._ptr(vamax), *ring_args(kv_cache), ops._stream())


def write(kv_cache, k, v, current_start, sink_tokens, local_attn_size, rope=None):
    """Store this forward's K/V, evicting the oldest non-sink tokens when the window is full
    (kv_cache.py:64-75). Returns (local_end_index, current_end). On the GPU the store and the block
    statistics are one kernel (`store`); `rope` (optional, GPU only) ropes K in that kernel, for a
    caller that would otherwise pass causal_rope_apply(k, rope)."""
    evicted, rolled, local_start_index, local_end_index, current_end = plan(
        kv_cache, k.shape[1], current_start, sink_tokens, local_attn_size)
    _ring_sink(kv_cache, sink_tokens)
    if evicted:
        evict(kv_cache, sink_tokens, evicted, rolled)
    if kv_cache["k"].is_cuda:
        store(kv_cache, k, v, local_start_index, rope)
        return local_end_index, current_end
    if rope is not None:
        raise ValueError("rope inside write is a GPU kernel; rope K on the host first")
    kv_cache["k"][:, local_start_index:local_end_index] = k
    kv_cache["v"][:, local_start_index:local_end_index] = v
    refresh_stats(kv_cache, local_start_index, local_end_index)
    return local_end_index, current_end


def window(kv_cache, local_end_index, max_attention_size):
    """The K/V slice this forward attends to (kv_cache.py:78-81). A ring cache returns the logical
    slice as a copy (the rows gathered in window order)."""
    start = max(0, local_end_index - max_attention_size)
    sink, rlen, head = ring_args(kv_cache)
    if rlen == 0 or head == 0:
        return kv_cache["k"][:, start:local_end_index], kv_cache["v"][:, start:local_end_index]
    t = torch.arange(start, local_end_index, device=kv_cache["k"].device)
    rows = torch.where(t < sink, t, sink + (t - sink + head) % rlen)
    return kv_cache["k"][:, rows], kv_cache["v"][:, rows]


def commit(kv_cache, current_end, local_end_index):
    kv_cache["global_end_int"] = current_end
    kv_cache["local_end_int"] = local_end_index
    kv_cache["global_end_index"].fill_(current_end)
    kv_cache["local_end_index"].fill_(local_end_index)


class WindowQuantizer:
    """Reusable device buffers for re-quantizing one cache window per call (no allocation per call
    once sized)."""

    def __init__(self):
        self.key = None

    def buffers(self, batch, heads, q_len, kv_len, device):
        key = (batch, heads, q_len, kv_len, str(device))
        if key != self.key:
            self.q_codes, self.q_scale = ops.alloc_q(batch, heads, q_len, device)
            (self.k_codes, self.k_scale, self.vt_codes, self.v_scale,
             self.km) = ops.alloc_kv(batch, heads, kv_len, 1, device)
            self.sums = torch.empty(batch * heads * 128 * 3, dtype=torch.float32, device=device)
            self.key = key
        return self


_default_quantizer = WindowQuantizer()


def quantize_window(q, kv_cache, end, quantizer=None, rope=None) -> ops.QuantWindow:
    """Quantize q and the cache window [0, end) with the cached block statistics
    (lbq_requant_cache + lbq_quant_q; with `rope` = the chunk's (cos, sin) tables, q is roped in the
    Q quantizer, lbq_rope_quant_q)."""
    k, v = kv_cache["k"], kv_cache["v"]
    ops._check_act("q", q)
    b, lq, h, _ = q.shape
    qz = (quantizer or _default_quantizer).buffers(b, h, lq, end, q.device)
    st = ops._stream()
    ksum, vamax = kv_cache["lbq_ksum"], kv_cache["lbq_vamax"]
    _lib.call("lbq_requant_cache", ops._ptr(k), *k.stride()[:3], ops._ptr(v), *v.stride()[:3], b, h, end,
              ksum.shape[1], ops._ptr(ksum), ops._ptr(vamax), ops._ptr(qz.sums), ops._ptr(qz.k_codes),
              ops._ptr(qz.k_scale), ops._ptr(qz.vt_codes), ops._ptr(qz.v_scale), ops._ptr(qz.km),
              *ring_args(kv_cache), st)
    if rope is None:
        _lib.call("lbq_quant_q", ops._ptr(q), *q.stride()[:3], b, h, lq, ops._ptr(qz.q_codes), ops._ptr(qz.q_scale),
                  st)
    else:
        rc, rs, sr_b, sr_l = _rope_args(rope)
        _lib.call("lbq_rope_quant_q", ops._ptr(q), *q.stride()[:3], rc, rs, sr_b, sr_l, b, h, lq,
                  ops._ptr(qz.q_codes), ops._ptr(qz.q_scale), st)
    return ops.QuantWindow(qz.q_codes, qz.q_scale, qz.k_codes, qz.k_scale, qz.vt_codes, qz.v_scale, qz.km, lq, end,
                           end, 1)


def attend(q, kv_cache, start, end, sm_scale=None, num_splits=None, out=None, quantizer=None, rope=None):
    """`sageattn(q, k_win, v_win, "NHD")` with the window [0, end) of `kv_cache`, whose tokens
    [start, end) were written by this forward — the role of sage_preq.attend (sage_preq.py:107-128).
    `start` is accepted for signature parity; the statistics were refreshed by `write`. With `rope`,
    q is the un-roped query and is roped in the Q quantizer."""
    w = quantize_window(q, kv_cache, end, quantizer, rope)
    return ops.attn_from_codes(w, sm_scale=sm_scale, out=out, num_splits=num_splits)
