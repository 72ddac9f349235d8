"""lbw_b200: B200-native (sm_100a) causal-fast DiT block forward of LingBot-World-v2.

Importable as `lbw_b200` once __graft_entry__ has registered this directory (its on-disk name,
lingbot-world-v2_b200, is not a Python identifier). Modules:
  _lib / kernels      C ABI (liblbw.so, include/lbw.h) and torch wrappers
  attention, ffn_mx   operators with the reference's names (wan/modules/attention.py, kernels/ffn_mx.py)
  block, model        drop-in CausalWanAttentionBlock, the N-block loop and CausalWanModel (WanModelFast)
  checkpoint          the reference's DiT checkpoint folder -> CausalWanModel
  chunked_kv_cache    chunk routing / cache allocation (wan/modules/chunked_kv_cache.py)
  rope, sp            RoPE tables; sequence-parallel token shards + K/V all-gather
  vae                 Wan 2.1 VAE decoder (wan/modules/vae2_1.py decode / decode_chunk)
"""
from . import _lib  # noqa: F401
