"""Sequence split of the DiT's self-attention across GPUs — replaces the head/token split of
lingbot/parallel/split_dit.py:366-445 and the head-divisibility rule of lingbot/parallel/config.py:13-17.

The reference splits attention heads across cards (Ulysses), so its degree must divide the 12 heads,
which 8 GPUs do not. Here every rank keeps all heads and a 128-row slice of the chunk's queries: query
rows are independent given the full key window. Projections are token-sharded, so each rank holds a
contiguous share of the current chunk's K/V; `gather_tokens` all-gathers it (NCCL over NVLink on the
GPU, gloo on the CPU) into the rank's replica of the cache. The memory part of the window is already
replicated on every rank: it was gathered when it was the current chunk.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

Q_ALIGN = 128   # query-slice granularity: whole 128-row Q tiles, so per-warp Q scales (32 rows) match


@dataclass(frozen=True)
class ParallelConfig:
    """How one run is laid out across GPUs (the role of lingbot/parallel/config.py:6-17).
    `sp` ranks split the query tokens; there is no head-divisibility requirement."""
    sp: int = 1

    @property
    def world_size(self):
        return self.sp

    def validate(self, num_heads, world_size):
        if self.world_size != world_size:
            raise ValueError(f"{self} needs {self.world_size} processes, got {world_size}")
        if self.sp < 1:
            raise ValueError(f"sequence split degree must be >= 1, got {self.sp}")
        if num_heads < 1:
            raise ValueError("need at least one attention head")


def shard_rows(q_len, world, rank, align=Q_ALIGN):
    """Rank `rank`'s query rows [r0, r1): 128-row tiles dealt out contiguously, the last rank taking the
    remainder (it may be empty when world > tiles)."""
    tiles = (q_len + align - 1) // align
    per = -(-tiles // world)
    r0 = min(q_len, rank * per * align)
    r1 = min(q_len, (rank + 1) * per * align)
    return r0, r1


def token_part(n, world):
    """Tokens per rank of a token-sharded chunk of n tokens (the last share is zero-padded)."""
    return -(-n // world)


def token_shard(n, world, rank):
    """Rank `rank`'s contiguous token share [lo, hi) of a chunk of n tokens."""
    part = token_part(n, world)
    lo = min(n, rank * part)
    return lo, min(n, lo + part)


def gather_tokens(x_part, n, group=None, out=None):
    """All-gather token shares [B, part, H, D] (zero-padded to `token_part(n, world)`) into the whole
    chunk [B, n, H, D], in token order (rank-major == token order)."""
    world = dist.get_world_size(group)
    b, part, h, d = x_part.shape
    if part != token_part(n, world):
        raise ValueError(f"share of {part} tokens, expected {token_part(n, world)} for n={n}, world={world}")
    buf = out if out is not None else torch.empty(world, b, part, h, d, dtype=x_part.dtype, device=x_part.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf, x_part.contiguous(), group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), x_part.contiguous(), group=group)
    return buf.permute(1, 0, 2, 3, 4).reshape(b, world * part, h, d)[:, :n]


def pad_share(x_full, world, rank, part=None):
    """This rank's zero-padded share [B, part, H, D] of a chunk [B, n, H, D] (test and bench helper);
    shares are `token_part` tokens unless `part` is given (e.g. `share_part`)."""
    b, n, h, d = x_full.shape
    part = token_part(n, world) if part is None else part
    lo = min(n, rank * part)
    hi = min(n, lo + part)
    share = torch.zeros(b, part, h, d, dtype=x_full.dtype, device=x_full.device)
    share[:, :hi - lo] = x_full[:, lo:hi]
    return share


def attend_split(q_rows, cache, k_part, v_part, current_start, sink_tokens, local_attn_size,
                 max_attention_size, n_tokens, group=None, sm_scale=None):
    """One rank's self-attention for a chunk: gather the chunk's K/V shares, write them into this rank's
    cache replica (kv_cache.write, which refreshes the block statistics), quantize the window and attend
    this rank's query rows `q_rows` [B, r1-r0, H, 128]. Returns (out_rows, local_end, current_end);
    the caller commits (kv_cache.commit) after the chunk's forward, as the reference does."""
    from . import kv_cache
    k = gather_tokens(k_part, n_tokens, group)
    v = gather_tokens(v_part, n_tokens, group)
    end, cur_end = kv_cache.write(cache, k, v, current_start, sink_tokens, local_attn_size)
    if end > max_attention_size:
        raise NotImplementedError("the window must start at token 0 of the cache (kv_size <= max_attention_size)")
    out = kv_cache.attend(q_rows, cache, end - n_tokens, end, sm_scale=sm_scale)
    return out, end, cur_end


def share_part(n, world, align=Q_ALIGN):
    """Tokens per rank of the peer-memory split: whole 128-token tiles, so that a rank's K/V share and
    its query slice (`shard_rows`) are the same tokens and every share starts on a 64-token K block."""
    tiles = (n + align - 1) // align
    return -(-tiles // world) * align


class SplitAttention:
    """One rank's sequence-split self-attention for one layer of a chunk, exchanging over NVLink peer
    memory (replaces the head split + host-staged q/k/v exchange of lingbot/parallel/split_dit.py:366-445).

    The window is the replicated memory part of the cache (tokens [0, mem_len)) plus the current chunk
    of n_tokens, token-sharded across ranks in `share_part` slices (rank r holds chunk tokens
    [r*part, (r+1)*part) as k/v shares, and attends the same query rows). Per call, on this rank:

      1. lbq_kv_block_stats   — block statistics of the share into this rank's cache tables;
      2. lbq_share_totals_push — the share's per-channel totals -> every rank's exchange area;
         lbq_chunk_totals     — wait for every rank's totals; window totals (memory + shares in rank
                                order, identical on every rank);
      3. quantize the memory segment (K mean-smoothed int8, V e4m3), while on a side stream
         lbq_share_push       — the bf16 share and its block statistics -> every rank's cache replica
                                and tables (forked after the totals push when the cache was last used two
                                or more calls ago, else after lbq_chunk_totals) and the query slice is
                                quantized;
      4. lbq_peer_wait        — wait for the other ranks' shares; quantize the chunk segment;
      5. attention over the two segments.

    A CUDA graph replays the launch order chosen at capture: replay per-cache calls in the order they
    were captured (as a layer loop does).

    Codes and scales are identical to quantizing the whole window in one piece (mem_len % 64 == 0
    keeps the 64-token K blocks those of the whole window). The caches must be carved from `heap`
    (kv_cache.allocate(..., heap=heap)), identically on every rank. Every launch is on the current
    stream (plus one forked side stream), without host synchronisation, so a call can be captured in
    a CUDA graph and replayed. `memory_changed(cache)` must be called whenever the memory part of a
    cache changes.
    """

    def __init__(self, batch, heads, q_rows, mem_len, n_tokens, device, heap, group=None, timeout_s=4.0):
        from . import _lib, ops
        if mem_len % 64:
            raise ValueError("the memory part must be a whole number of 64-token blocks")
        if 0 < mem_len < n_tokens:
            raise ValueError("the chunk segment cannot be longer than the memory segment")
        self.group, self.heap = group, heap
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if heap.world != self.world or heap.rank != self.rank:
            raise ValueError("the peer heap was built for another group")
        self.b, self.h, self.q_rows = batch, heads, q_rows
        self.mem_len, self.n = mem_len, n_tokens
        self.part = share_part(n_tokens, self.world)
        self.nb_part = self.part // 64
        lo = min(n_tokens, self.rank * self.part)
        self.share_valid = min(n_tokens, lo + self.part) - lo
        self.lo = lo
        self.timeout_ns = int(timeout_s * 1e9)
        cols = batch * heads * 128
        xbytes = _lib.load().lbq_exchange_bytes(self.world, batch, heads)
        if xbytes <= 0:
            raise ValueError(f"no exchange layout for {self.world} ranks")
        self.xchg = heap.carve((xbytes,), torch.uint8)          # zeroed; caller barriers before first use
        self.xchg_off = heap.offset(self.xchg)
        self.q_codes, self.q_scale = ops.alloc_q(batch, heads, max(q_rows, 1), device)
        (self.k_codes, self.k_scale, self.vt_codes, self.v_scale,
         self.km) = ops.alloc_kv(batch, heads, mem_len, 2, device)
        self.tot_ksum = torch.zeros(cols, dtype=torch.float64, device=device)
        self.tot_vamax = torch.zeros(cols, dtype=torch.float32, device=device)
        self.side = torch.cuda.Stream(device=device)
        self.fork, self.join = torch.cuda.Event(), torch.cuda.Event()
        self._calls = 0
        self._last_use = {}      # id(cache) -> index of the call that last used it
        self.push_ctas = 64      # CTAs of the share push (measured best beside the quantizers); the same
                                 # on every rank
        self.early_push = False  # fork the share push before the totals wait (when the cache allows it);
                                 # off: the bulk push then delays the tagged totals on NVLink

    def memory_changed(self, cache):
        """Per-channel totals of the memory part from the cache's block statistics, kept in the cache
        dict (one SplitAttention, i.e. one set of code buffers, can serve every layer)."""
        from . import _lib, ops
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        cols = self.b * self.h * 128
        if "lbq_mem_ksum" not in cache:
            cache["lbq_mem_ksum"] = torch.zeros(cols, dtype=torch.float64, device=ksum.device)
            cache["lbq_mem_vamax"] = torch.zeros(cols, dtype=torch.float32, device=ksum.device)
        if self.mem_len == 0:
            cache["lbq_mem_ksum"].zero_()
            cache["lbq_mem_vamax"].zero_()
            return
        _lib.call("lbq_kv_window_sums", ops._ptr(ksum), ops._ptr(vamax), self.b, self.h, 0, self.mem_len // 64,
                  ksum.shape[1], ops._ptr(cache["lbq_mem_ksum"]), ops._ptr(cache["lbq_mem_vamax"]), ops._stream())

    def _check_cache(self, cache):
        k = cache["k"]
        b, lk, h, d = k.shape
        if (b, h, d) != (self.b, self.h, 128) or not (k.is_contiguous() and cache["v"].is_contiguous()):
            raise ValueError("cache K/V must be contiguous [B, tokens, H, 128] buffers of this split")
        if lk < self.mem_len + self.n:
            raise ValueError(f"cache of {lk} tokens cannot hold {self.mem_len} memory + {self.n} chunk tokens")
        return self.heap.offset(k), self.heap.offset(cache["v"]), lk

    def __call__(self, q_rows, cache, k_part, v_part, out, sm_scale=None, num_splits=None, attn_events=None):
        """q_rows [B, rows, H, 128] (this rank's query slice), k_part/v_part [B, part, H, 128] (this rank's
        share of the chunk, rows past the chunk's end ignored) -> out [B, rows, H, 128]; also writes the
        whole chunk into `cache` at [mem_len, mem_len + n_tokens) and its block statistics, as
        kv_cache.write does."""
        from . import _lib, ops
        st = torch.cuda.current_stream()
        stp = st.cuda_stream
        b, h = self.b, self.h
        if k_part.shape[1] < self.share_valid or v_part.shape[1] < self.share_valid:
            raise ValueError(f"shares of {k_part.shape[1]} tokens, expected {self.part}")
        k_off, v_off, lk = self._check_cache(cache)
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        max_blocks = ksum.shape[1]
        row0 = (self.mem_len + self.lo) // 64
        nb_valid = (self.share_valid + 63) // 64
        peers = ops._ptr(self.heap.peers)
        group = (peers, self.world, self.rank, self.xchg_off)
        share = (ops._ptr(k_part), *k_part.stride()[:3], ops._ptr(v_part), *v_part.stride()[:3])
        # 1. block statistics of the share into this rank's tables
        if nb_valid > 0:
            _lib.call("lbq_kv_block_stats", *share, b, h, self.share_valid, 0, nb_valid, max_blocks,
                      ksum.data_ptr() + row0 * h * 128 * 8, vamax.data_ptr() + row0 * h * 128 * 4, stp)
        # 2. the share's totals -> every rank (before the bulk push, so that they do not queue behind it)
        _lib.call("lbq_share_totals_push", ops._ptr(ksum), ops._ptr(vamax), max_blocks, row0, nb_valid, b, h,
                  *group, stp)
        # the share push may start now unless a rank could still be reading this cache's chunk region:
        # every rank has started the previous call (its totals signal was consumed by the previous call's
        # lbq_chunk_totals), so a cache last used two or more calls ago is free
        last = self._last_use.get(id(cache))
        early = self.early_push and last is not None and self._calls - last >= 2
        self._last_use[id(cache)] = self._calls
        self._calls += 1
        kv_len = self.mem_len + self.n
        rows = q_rows.shape[1]

        def side_work():
            # the bf16 share (+ its block statistics) -> every rank; the query slice's codes
            self.fork.record(st)
            self.side.wait_event(self.fork)
            _lib.call("lbq_share_push", *share, b, h, self.share_valid, self.nb_part, *group, k_off, v_off, lk,
                      self.mem_len + self.lo, self.heap.offset(ksum), self.heap.offset(vamax), max_blocks,
                      self.push_ctas, self.side.cuda_stream)
            if rows > 0:
                _lib.call("lbq_quant_q", ops._ptr(q_rows), *q_rows.stride()[:3], b, h, rows, ops._ptr(self.q_codes),
                          ops._ptr(self.q_scale), self.side.cuda_stream)
            self.join.record(self.side)

        if early:
            side_work()
        # every rank's totals -> the window totals (identical on every rank)
        _lib.call("lbq_chunk_totals", *group, b, h, ops._ptr(cache["lbq_mem_ksum"]), ops._ptr(cache["lbq_mem_vamax"]),
                  ops._ptr(self.tot_ksum), ops._ptr(self.tot_vamax), self.timeout_ns, stp)
        if not early:
            side_work()
        # 3. the memory segment is quantized while the shares travel
        kc, vc = cache["k"], cache["v"]
        codes = (ops._ptr(self.tot_ksum), ops._ptr(self.tot_vamax), ops._ptr(self.k_codes), ops._ptr(self.k_scale),
                 ops._ptr(self.vt_codes), ops._ptr(self.km), ops._ptr(self.v_scale))
        src = (ops._ptr(kc), *kc.stride()[:3], ops._ptr(vc), *vc.stride()[:3], b, h)
        nseg = 2 if self.mem_len > 0 else 1
        seg_len = self.mem_len if self.mem_len > 0 else self.n
        if self.mem_len > 0:
            _lib.call("lbq_quant_kv", *src, 0, 0, 2, self.mem_len, self.mem_len, kv_len, *codes, 1, stp)
        # 4. every share has landed: quantize the chunk segment
        st.wait_event(self.join)
        _lib.call("lbq_peer_wait", *group, self.nb_part, b, h, self.push_ctas, self.timeout_ns, stp)
        _lib.call("lbq_quant_kv", *src, self.mem_len, nseg - 1, nseg, self.n, seg_len, kv_len, *codes,
                  int(self.mem_len == 0), stp)
        if rows == 0:
            return out
        w = ops.QuantWindow(self.q_codes, self.q_scale, self.k_codes, self.k_scale, self.vt_codes, self.v_scale,
                            self.km, rows, kv_len, seg_len, nseg)
        if attn_events is not None:
            attn_events[0].record()
        ops.attn_from_codes(w, sm_scale=sm_scale, out=out, num_splits=num_splits)
        if attn_events is not None:
            attn_events[1].record()
        return out

    def launches(self, num_splits):
        """Our kernels per call: share block stats, totals push, window totals, share push, memory K/V
        quantizer, Q quantizer, peer wait, chunk K/V quantizer, attention (+ split-KV combine)."""
        return (1 + 2 + 1 + (1 if self.mem_len > 0 else 0) + (1 if self.q_rows > 0 else 0) + 1 + 1 + 1
                + (1 if num_splits > 1 else 0))
