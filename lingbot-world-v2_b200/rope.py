"""3-D RoPE tables for the B200 kernels.

The reference rotates interleaved (re, im) pairs of each 128-wide head with angles split
22 / 21 / 21 pairs over (frame, height, width) (wan/modules/model_fast.py:878-931, :933-979;
freqs built at :3273-3278 from rope_params, wan/modules/model.py:47-53). Its grids are full
[L, 1, 64] cos/sin tensors; the rmsnorm_rope kernel instead takes the three small factor tables
(frames of this chunk x 22, grid_h x 21, grid_w x 21) and indexes them per token, so only
(f + h + w) x 21-22 values cross to the device. The angles are the same fp32 products and cos/sin
are taken on the CPU in fp32 exactly as the reference does, so the tables are bit-identical to the
reference grids' entries.
"""
import torch

HEAD_DIM = 128

# Arithmetic of the rotation, process-wide as in the reference (model_fast.py:985-1003): fp32 until a model forward
# sees a chunk of 4,096 or more tokens, bf16 from then on (cos / sin rounded to bf16 and every product and sum of the
# rotation rounded to bf16: lbw.h LBW_ROPE_BF16). The block reads it at each call.
ROPE_DTYPE = torch.float32


def mark_bf16_rope():
    """bf16 RoPE for the rest of this process (model_fast.py:1000-1003)."""
    global ROPE_DTYPE
    ROPE_DTYPE = torch.bfloat16


def set_bf16_rope_for_forward(seq_len):
    """Called once per model forward with its seq_len, as the reference does (model_fast.py:1144-1148, :3348)."""
    if seq_len >= 4096:
        mark_bf16_rope()


def rope_params(max_seq_len, dim, theta=10000):
    pos = torch.arange(max_seq_len).float()
    inv = 1.0 / torch.pow(theta, torch.arange(0, dim, 2).float().div(dim))
    return torch.outer(pos, inv)


def rope_freqs(head_dim=HEAD_DIM, max_frames=2880):
    """[max_frames, head_dim / 2] angle table (frame part | height part | width part)."""
    d = head_dim
    dt = d - 4 * (d // 6)
    return torch.cat([rope_params(max_frames, dt), rope_params(max_frames, 2 * (d // 6)),
                      rope_params(max_frames, 2 * (d // 6))], dim=1)


def split_sizes(freqs):
    c = freqs.shape[1]
    return c - 2 * (c // 3), c // 3


_CACHE = {}


def rope_tables(freqs, grid, start_frame, device):
    """(cos, sin) fp32 device tables [f*22 + h*21 + w*21] for a chunk of grid (f, h, w) whose first
    frame is `start_frame` (= current_start // frame_seqlen)."""
    f, h, w = (int(v) for v in grid)
    if torch.compiler.is_compiling():   # no host-side cache inside a traced graph
        return _tables(freqs, f, h, w, int(start_frame), device)
    key = (id(freqs), tuple(freqs.shape), f, h, w, int(start_frame), str(device))
    hit = _CACHE.get(key)
    if hit is not None and hit[0] is freqs:
        return hit[1]
    out = _tables(freqs, f, h, w, int(start_frame), device)
    _CACHE[key] = (freqs, out)
    return out


def _tables(freqs, f, h, w, start_frame, device):
    fc = freqs.detach().cpu().float()
    s0, s1 = split_sizes(fc)
    if (s0, s1) != (22, 21):
        raise ValueError(f"rope tables are laid out for head_dim 128 (22/21/21 pairs), got {s0}/{s1}/{s1}")
    ang = torch.cat([fc[start_frame:start_frame + f, :s0].reshape(-1), fc[:h, s0:s0 + s1].reshape(-1),
                     fc[:w, s0 + s1:].reshape(-1)])
    return torch.cos(ang).to(device), torch.sin(ang).to(device)
