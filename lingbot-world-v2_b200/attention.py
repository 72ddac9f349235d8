"""Attention operators with the reference's names and argument meaning (wan/modules/attention.py),
served by the sm_100a chunk-attention kernel (liblbw.so: lbw_chunk_attention).

  exact_attention_chunks(q, k_chunks, v_chunks)   attention.py:1048-1058
  attention(q, k, v, ...)                         attention.py:1082-1143 (non-causal, no mask)
  const_max_ag_attention(q, k_shard, v_shard, k_chunks, v_chunks)
                                                  attention.py:248-265 -- here exact softmax, and the
                                                  shard all-gather into the destination chunk is done
                                                  over NCCL by lbw_b200.sp (or written locally at P=1)
  cross_dedup_bias(k, v, kc)                      attention.py:516-523
  cross_attention_dedup(q, k, v, bias, kc)        attention.py:532-554 (token-major K/V here)

q/k/v are [1, L, n, d] (or [L, n, d]) bf16 CUDA tensors with d = 128; outputs are [1, Lq, n, d] bf16.
"""
import torch

from . import kernels


def _lq(q):
    return q.shape[-3]


def exact_attention_chunks(q, k_chunks, v_chunks, dtype=torch.bfloat16):
    if dtype != torch.bfloat16:
        raise ValueError("the B200 attention kernel produces bf16")
    out = kernels.chunk_attention(q.contiguous(), [k.contiguous() for k in k_chunks],
                                  [v.contiguous() for v in v_chunks])
    return out.view(1, _lq(q), q.shape[-2], q.shape[-1])


def exact_attention(q, k, v, dtype=torch.bfloat16):
    return exact_attention_chunks(q, [k], [v], dtype=dtype)


def attention(q, k, v, q_lens=None, k_lens=None, dropout_p=0.0, softmax_scale=None, q_scale=None, causal=False,
              window_size=(-1, -1), deterministic=False, dtype=torch.bfloat16, fa_version=None, attn_mask=None,
              is_cross_attn=False, kv_lo=None, kv_hi=None):
    if causal or attn_mask is not None or dropout_p or kv_lo is not None or kv_hi is not None:
        raise ValueError("the chunked cache path needs no mask: causal/attn_mask/kv bounds are not supported")
    if q_scale is not None:
        q = (q.float() * q_scale).to(q.dtype)
    out = kernels.chunk_attention(q.contiguous(), [k.contiguous()], [v.contiguous()], softmax_scale=softmax_scale)
    return out.view(1, _lq(q), q.shape[-2], q.shape[-1]).to(dtype)


flash_attention = attention


def const_max_ag_attention(q, k_shard, v_shard, k_chunks, v_chunks):
    """Exact attention over (leading..., destination). The destination chunk receives this rank's
    K/V shard (gathered over the sequence-parallel group when one is set); returns
    (out, k_dest, v_dest) like the reference."""
    from . import sp
    k_dest, v_dest = k_chunks[-1], v_chunks[-1]
    sp.write_and_gather(k_shard, k_dest)
    sp.write_and_gather(v_shard, v_dest)
    return exact_attention_chunks(q, k_chunks, v_chunks), k_dest, v_dest


fa2_ag_attention = const_max_ag_attention


def cross_dedup_bias(k, v, kc):
    """log(m / r) on the r rows among the first kc equal to the last row of both K and V (m such rows
    in total), 0 elsewhere. Runs once per generation when the cross cache is filled."""
    k2 = k.reshape(k.shape[-3], -1)
    v2 = v.reshape(v.shape[-3], -1)
    same = (k2 == k2[-1:]).all(dim=1) & (v2 == v2[-1:]).all(dim=1)
    s = same[:kc]
    m, r = same.sum().float(), s.sum().float()
    return torch.where(s, torch.log(m / r.clamp(min=1)), torch.zeros((), dtype=torch.float32, device=k.device))


def cross_attention_dedup(q, k, v, bias, kc, dtype=torch.bfloat16):
    """q [1, Lq, n, d] against the first kc keys of the cross cache with the per-key bias.
    k/v: token-major [1, T, n, d] or [T, n, d]."""
    k2 = k.reshape(-1, k.shape[-2], k.shape[-1])[:kc].contiguous()
    v2 = v.reshape(-1, v.shape[-2], v.shape[-1])[:kc].contiguous()
    out = kernels.chunk_attention(q.contiguous(), [k2], [v2], key_bias=bias.float().contiguous())
    return out.view(1, _lq(q), q.shape[-2], q.shape[-1]).to(dtype)
