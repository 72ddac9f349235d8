"""lbw_b200: B200-native (sm_100a) causal-fast DiT block forward of LingBot-World-v2.

Importable as `lbw_b200` once __graft_entry__ has registered this directory (its on-disk name,
lingbot-world-v2_b200, is not a Python identifier). Modules:
  _lib / kernels      C ABI (liblbw.so, include/lbw.h) and torch wrappers
  attention, ffn_mx   operators with the reference's names (wan/modules/attention.py, kernels/ffn_mx.py)
  block, model        drop-in CausalWanAttentionBlock and the N-block loop
  chunked_kv_cache    chunk routing / cache allocation (wan/modules/chunked_kv_cache.py)
  rope, sp            RoPE tables; sequence-parallel token shards + K/V all-gather
"""
from . import _lib  # noqa: F401
