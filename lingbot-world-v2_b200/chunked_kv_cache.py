"""Chunked KV cache: per-block lists of independent K/V chunk tensors.

Same contract as the reference's wan/modules/chunked_kv_cache.py: chunk 0 is the pinned sink,
the others are destinations in round-robin order, and each forward sees its chunks ordered
(leading..., destination) with the destination LAST. The B200 kernels read the token-major layout
[B, chunk_tokens, N, D] (TMA tiles of 128 tokens x 128 head dims); the N-major layouts of the
Trainium const-max kernels are not used.
"""
import torch


def num_chunks(local_attn_size, chunk_size):
    """Window chunks = local_attn_size // chunk_size (0 for a global cache). Reference :35-44."""
    if local_attn_size is None or local_attn_size < 0:
        return 0
    return max(1, int(local_attn_size) // max(1, int(chunk_size)))


def chunk_routing(chunk_index, n_chunks):
    """(destination, leading) for the write of chunk `chunk_index` (reference :47-76).

    Chunk 0 is written once (the sink); later chunks rotate through slots 1..n_chunks-1. The leading
    tuple lists the slots already holding data, in slot order, without the destination."""
    i = int(chunk_index)
    if n_chunks <= 1:
        return 0, ()
    if i == 0:
        dest = 0
    else:
        dest = 1 + (i - 1) % (n_chunks - 1)
    filled = i if i < n_chunks else n_chunks
    return dest, tuple(s for s in range(filled) if s != dest)


def allocate_self_kv_chunks(num_layers, batch, chunk_tokens, heads, head_dim, n_chunks, dtype, device,
                            n_major=False, own_tokens=0):
    """Per block {'k': [n_chunks x [B, chunk_tokens, N, D]], 'v': [...]}, independent zeroed tensors
    (reference :79-169)."""
    if n_major is not False and (n_major is True or any(n_major)):
        raise ValueError("the B200 chunk-attention kernel reads the token-major [B, L, N, D] layout only")
    if own_tokens:
        raise ValueError("own-shard chunk copies (LINGBOT_ATTN_SPLIT) are not used by the B200 path")
    cache = []
    for _ in range(num_layers):
        ks = [torch.zeros(batch, chunk_tokens, heads, head_dim, dtype=dtype, device=device) for _ in range(n_chunks)]
        vs = [torch.zeros(batch, chunk_tokens, heads, head_dim, dtype=dtype, device=device) for _ in range(n_chunks)]
        cache.append({"k": ks, "v": vs})
    return cache


def ordered_chunks(block_cache, destination, leading):
    order = (*leading, destination)
    return tuple(block_cache["k"][i] for i in order), tuple(block_cache["v"][i] for i in order)


def ordered_chunks_by_block(cache, destination, leading):
    pairs = [ordered_chunks(bc, destination, leading) for bc in cache]
    return tuple(p[0] for p in pairs), tuple(p[1] for p in pairs)


def chunk_bytes(cache):
    return sum(t.numel() * t.element_size() for bc in cache for key in ("k", "v") for t in bc.get(key, ()))
