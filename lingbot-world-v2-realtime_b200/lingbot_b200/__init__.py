"""lingbot_b200 — the quantized (INT8 QK^T / FP8 PV) self-attention path of the LingBot-World causal
DiT, rebuilt for B200 (sm_100a) behind a C ABI (liblbq.so, include/lbq.h).

Public surface (mirrors the reference's modules of the same role):
  attention.attention   drop-in for lingbot/layers/attention.py:attention
  kv_cache              drop-in for lingbot/layers/kv_cache.py, plus the quantized-window attend
                        that replaces lingbot/layers/sage_preq.py:attend
  split                 sequence split across GPUs (replaces lingbot/parallel/split_dit.py's
                        exchange and the head-divisibility rule of lingbot/parallel/config.py)
"""
__all__ = ["attention", "kv_cache", "ops", "split"]
