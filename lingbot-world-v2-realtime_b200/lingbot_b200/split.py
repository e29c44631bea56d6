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


def pad_share(x_full, world, rank):
    """This rank's zero-padded share [B, part, H, D] of a chunk [B, n, H, D] (test and bench helper)."""
    b, n, h, d = x_full.shape
    part = token_part(n, world)
    lo, hi = token_shard(n, world, rank)
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


class SplitAttention:
    """One rank's sequence-split self-attention for one layer of a chunk, with the exchange overlapped.

    The window is the replicated memory part of the cache (tokens [0, mem_len)) plus the current chunk
    (n_tokens, token-sharded across ranks). The K mean and V absmax of the window only need per-channel
    totals, so each rank reduces its own share of the chunk, the totals are all-reduced (12 bytes per
    channel), and the memory part is quantized while the bf16 all-gather of the chunk is in flight; the
    chunk is quantized once it lands. The window is handed to the attention kernel as two KV segments
    (memory, chunk), which requires mem_len % 64 == 0 so that the 64-token K blocks are those of the
    whole window; codes and scales are then identical to quantizing the window in one piece.
    `memory_changed(cache)` must be called whenever the memory part of the cache changes (after a
    chunk's memory-write pass).
    """

    def __init__(self, batch, heads, q_rows, mem_len, n_tokens, device, group=None):
        from . import ops
        if mem_len % 64:
            raise ValueError("the memory part must be a whole number of 64-token blocks")
        self.group = group
        self.world = dist.get_world_size(group)
        self.b, self.h, self.q_rows = batch, heads, q_rows
        self.mem_len, self.n = mem_len, n_tokens
        self.part = token_part(n_tokens, self.world)
        rank = dist.get_rank(group)
        lo, hi = token_shard(n_tokens, self.world, rank)
        self.share_valid = hi - lo
        cols = batch * heads * 128
        self.q_codes, self.q_scale = ops.alloc_q(batch, heads, max(q_rows, 1), device)
        (self.k_codes, self.k_scale, self.vt_codes, self.v_scale,
         self.km) = ops.alloc_kv(batch, heads, mem_len, 2, device)
        nb = max(1, (self.part + 63) // 64)
        self.share_ksum = torch.zeros(batch, nb, heads, 128, dtype=torch.float64, device=device)
        self.share_vamax = torch.zeros(batch, nb, heads, 128, dtype=torch.float32, device=device)
        self.cur_ksum = torch.zeros(cols, dtype=torch.float64, device=device)
        self.cur_vamax = torch.zeros(cols, dtype=torch.float32, device=device)
        self.tot_ksum = torch.zeros(cols, dtype=torch.float64, device=device)
        self.tot_vamax = torch.zeros(cols, dtype=torch.float32, device=device)
        self.gather = torch.empty(2, self.world, batch, self.part, heads, 128, dtype=torch.bfloat16, device=device)

    def memory_changed(self, cache):
        """Per-channel totals of the memory part from the cache's block statistics, kept in the cache
        dict (one SplitAttention, i.e. one set of code buffers, can serve every layer)."""
        from . import _lib, ops
        ksum, vamax = cache["lbq_ksum"], cache["lbq_vamax"]
        cols = self.b * self.h * 128
        if "lbq_mem_ksum" not in cache:
            cache["lbq_mem_ksum"] = torch.zeros(cols, dtype=torch.float64, device=ksum.device)
            cache["lbq_mem_vamax"] = torch.zeros(cols, dtype=torch.float32, device=ksum.device)
        _lib.call("lbq_kv_window_sums", ops._ptr(ksum), ops._ptr(vamax), self.b, self.h, 0, self.mem_len // 64,
                  ksum.shape[1], ops._ptr(cache["lbq_mem_ksum"]), ops._ptr(cache["lbq_mem_vamax"]), ops._stream())

    def __call__(self, q_rows, cache, k_part, v_part, out, sm_scale=None, num_splits=None, attn_events=None):
        """q_rows [B, rows, H, 128] (this rank's query slice), k_part/v_part [B, part, H, 128] (this rank's
        zero-padded share of the chunk) -> out [B, rows, H, 128]; also writes the chunk into `cache` at
        [mem_len, mem_len + n_tokens) and refreshes its block statistics, as kv_cache.write does."""
        from . import _lib, kv_cache, ops
        st = ops._stream()
        b, h = self.b, self.h
        # 1. this rank's share totals -> all-reduced chunk totals
        if self.share_valid > 0:
            nb = (self.share_valid + 63) // 64
            _lib.call("lbq_kv_block_stats", ops._ptr(k_part), *k_part.stride()[:3], ops._ptr(v_part),
                      *v_part.stride()[:3], b, h, self.share_valid, 0, nb, self.share_ksum.shape[1],
                      ops._ptr(self.share_ksum), ops._ptr(self.share_vamax), st)
            _lib.call("lbq_kv_window_sums", ops._ptr(self.share_ksum), ops._ptr(self.share_vamax), b, h, 0, nb,
                      self.share_ksum.shape[1], ops._ptr(self.cur_ksum), ops._ptr(self.cur_vamax), st)
        else:
            self.cur_ksum.zero_()
            self.cur_vamax.zero_()
        dist.all_reduce(self.cur_ksum, op=dist.ReduceOp.SUM, group=self.group)
        dist.all_reduce(self.cur_vamax, op=dist.ReduceOp.MAX, group=self.group)
        # 2. the chunk's bf16 K/V travel while the memory part is quantized
        kw = dist.all_gather_into_tensor(self.gather[0], k_part.contiguous(), group=self.group, async_op=True)
        vw = dist.all_gather_into_tensor(self.gather[1], v_part.contiguous(), group=self.group, async_op=True)
        torch.add(cache["lbq_mem_ksum"], self.cur_ksum, out=self.tot_ksum)
        torch.maximum(cache["lbq_mem_vamax"], self.cur_vamax, out=self.tot_vamax)
        kv_len = self.mem_len + self.n
        kc, vc = cache["k"], cache["v"]
        common = (b, h)
        _lib.call("lbq_quant_kv", ops._ptr(kc), *kc.stride()[:3], ops._ptr(vc), *vc.stride()[:3], *common, 0, 0, 2,
                  self.mem_len, self.mem_len, kv_len, ops._ptr(self.tot_ksum), ops._ptr(self.tot_vamax),
                  ops._ptr(self.k_codes), ops._ptr(self.k_scale), ops._ptr(self.vt_codes), ops._ptr(self.km),
                  ops._ptr(self.v_scale), 1, st)
        rows = q_rows.shape[1]
        if rows > 0:
            _lib.call("lbq_quant_q", ops._ptr(q_rows), *q_rows.stride()[:3], b, h, rows, ops._ptr(self.q_codes),
                      ops._ptr(self.q_scale), st)
        kw.wait()
        vw.wait()
        kcur = self.gather[0].permute(1, 0, 2, 3, 4).reshape(b, self.world * self.part, h, 128)[:, :self.n]
        vcur = self.gather[1].permute(1, 0, 2, 3, 4).reshape(b, self.world * self.part, h, 128)[:, :self.n]
        # 3. the chunk: into the cache (for when it becomes memory) and into segment 1 of the codes
        kc[:, self.mem_len:kv_len] = kcur
        vc[:, self.mem_len:kv_len] = vcur
        kv_cache.refresh_stats(cache, self.mem_len, kv_len)
        _lib.call("lbq_quant_kv", ops._ptr(kc), *kc.stride()[:3], ops._ptr(vc), *vc.stride()[:3], *common,
                  self.mem_len, 1, 2, self.n, self.mem_len, kv_len, ops._ptr(self.tot_ksum),
                  ops._ptr(self.tot_vamax), ops._ptr(self.k_codes), ops._ptr(self.k_scale), ops._ptr(self.vt_codes),
                  ops._ptr(self.km), ops._ptr(self.v_scale), 0, st)
        if rows == 0:
            return out
        w = ops.QuantWindow(self.q_codes, self.q_scale, self.k_codes, self.k_scale, self.vt_codes, self.v_scale,
                            self.km, rows, kv_len, self.mem_len, 2)
        if attn_events is not None:
            attn_events[0].record()
        ops.attn_from_codes(w, sm_scale=sm_scale, out=out, num_splits=num_splits)
        if attn_events is not None:
            attn_events[1].record()
        return out
