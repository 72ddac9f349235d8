"""Sequence (context) parallelism of the block: flat token shards + the K/V all-gather.

The reference's deployed CP mode (LINGBOT_CP_FLAT_SEQ=1, wan/modules/model_fast.py:1042-1079,
:2066-2108) gives rank r the contiguous run [r*L/P, (r+1)*L/P) of the chunk's frame-major tokens.
Every per-token op (norms, projections, FFN, cross-attention, FiLM) stays local; the one exchange is
the all-gather of the new chunk's K and V shards into every rank's destination chunk, in rank order,
so the cached chunks are replicated. Attention is not token-causal, so the local queries against the
full window are exact with no softmax reduction across ranks.

The gather is one in-place ncclAllGather per tensor (torch.distributed over NCCL; gloo in the CPU
tests) on the destination chunk viewed as [chunk_tokens, C].
"""
import torch
import torch.distributed as dist

_GROUP = None
_ACTIVE = False


def set_group(group=None, enable=True):
    """Shard the blocks' tokens over `group` (None = the default group) when enable is True."""
    global _GROUP, _ACTIVE
    _GROUP, _ACTIVE = group, bool(enable)


def active():
    return _ACTIVE and dist.is_available() and dist.is_initialized() and world() > 1


def world():
    return dist.get_world_size(_GROUP) if dist.is_initialized() else 1


def rank():
    return dist.get_rank(_GROUP) if dist.is_initialized() else 0


def shard_range(n_tokens, r=None, p=None):
    """[start, end) of rank r's contiguous token run; n_tokens must divide evenly."""
    p = world() if p is None else p
    r = rank() if r is None else r
    if n_tokens % p:
        raise ValueError(f"{n_tokens} tokens do not split evenly over {p} ranks")
    n = n_tokens // p
    return r * n, (r + 1) * n


def shard_tokens(x, dim=0):
    if not active():
        return x
    a, b = shard_range(x.shape[dim])
    return x.narrow(dim, a, b - a)


def gather_tokens(x, dim=0):
    """Inverse of shard_tokens: concatenate the ranks' runs along `dim`."""
    if not active():
        return x
    xs = x.movedim(dim, 0).contiguous()
    out = torch.empty((xs.shape[0] * world(),) + tuple(xs.shape[1:]), dtype=xs.dtype, device=xs.device)
    dist.all_gather_into_tensor(out, xs, group=_GROUP)
    return out.movedim(0, dim)


def gather_rows_inplace(dest2d, local_rows):
    """dest2d [P * local_rows, C]: rank r's rows [r*local_rows, (r+1)*local_rows) are filled; gather all."""
    if not active():
        return dest2d
    r = rank()
    if dest2d.shape[0] != local_rows * world():
        raise ValueError(f"destination chunk has {dest2d.shape[0]} rows, expected {local_rows} x {world()}")
    mine = dest2d[r * local_rows:(r + 1) * local_rows]
    if dist.get_backend(_GROUP) != "nccl":
        mine = mine.clone()
    dist.all_gather_into_tensor(dest2d, mine, group=_GROUP)
    return dest2d


def write_and_gather(shard, dest):
    """Write this rank's shard [L/P, n, d] into its rows of dest [1, L, n, d] and gather the rest."""
    d2 = dest.view(-1, dest.shape[-2] * dest.shape[-1])
    s2 = shard.reshape(-1, d2.shape[1])
    a = rank() * s2.shape[0] if active() else 0
    d2[a:a + s2.shape[0]].copy_(s2)
    gather_rows_inplace(d2, s2.shape[0])
    return dest
