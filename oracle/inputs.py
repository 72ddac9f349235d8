"""Seeded synthetic inputs for one block (TEST INFRASTRUCTURE ONLY, see oracle/__init__.py).

Distributions follow the benchmark definition: Linear weights and biases ~N(0, 0.02); RMSNorm
gammas and the norm3 affine ~N(0, 0.02) ("flat" scores) or 1 + N(0, 0.02) ("peaked", which
exercises the online softmax max); adaLN modulation and e0 ~N(0, 0.1); x ~N(0, 1) rounded to bf16
and kept fp32; KV-cache entries and the text context ~N(0, 1) bf16; hoisted camera FiLM
scale/shift ~N(0, 0.1) bf16. Everything is drawn from numpy's PCG64 so the same seed gives the
same tensors on any machine.
"""
from dataclasses import dataclass, field

import numpy as np
import torch

HEAD_DIM = 128


@dataclass
class BlockCase:
    dim: int = 256
    ffn: int = 512
    grid: tuple = (3, 4, 6)        # (frames, h, w) of the query chunk
    n_lead: int = 2                # leading cache chunks (each one chunk of grid tokens)
    lead_rows: tuple = ()          # override per-chunk lengths of the leading chunks
    text_len: int = 32
    start_frame: int = 6
    peaked: bool = False
    film: bool = True
    dedup_rows: int = 0            # >0: context rows >= this are identical (cross_dedup input)
    cam: bool = False              # also draw the camera-FiLM MLP weights and a camera condition (last)
    seed: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def heads(self):
        return self.dim // HEAD_DIM

    @property
    def lq(self):
        f, h, w = self.grid
        return f * h * w


def _n(rng, shape, std, mean=0.0):
    return torch.from_numpy((rng.standard_normal(shape) * std + mean).astype(np.float32))


def make_params(case: BlockCase, rng):
    C, Fd = case.dim, case.ffn
    bf = torch.bfloat16
    p = {}
    for blk in ("self_attn", "cross_attn"):
        for nm in ("q", "k", "v", "o"):
            p[f"{blk}.{nm}.weight"] = _n(rng, (C, C), 0.02).to(bf)
            p[f"{blk}.{nm}.bias"] = _n(rng, (C,), 0.02).to(bf)
        g_mean = 1.0 if case.peaked else 0.0
        p[f"{blk}.norm_q.weight"] = _n(rng, (C,), 0.02, g_mean).to(bf)
        p[f"{blk}.norm_k.weight"] = _n(rng, (C,), 0.02, g_mean).to(bf)
    n3_mean = 1.0 if case.peaked else 0.0
    p["norm3.weight"] = _n(rng, (C,), 0.02, n3_mean).to(bf).float()
    p["norm3.bias"] = _n(rng, (C,), 0.02).to(bf).float()
    p["ffn.0.weight"] = _n(rng, (Fd, C), 0.02).to(bf)
    p["ffn.0.bias"] = _n(rng, (Fd,), 0.02).to(bf)
    p["ffn.2.weight"] = _n(rng, (C, Fd), 0.02).to(bf)
    p["ffn.2.bias"] = _n(rng, (C,), 0.02).to(bf)
    p["modulation"] = _n(rng, (1, 6, C), 0.1)
    return p


def make_case(case: BlockCase):
    """Returns (params, inputs) as CPU tensors."""
    rng = np.random.Generator(np.random.PCG64(case.seed))
    p = make_params(case, rng)
    C, H, Lq = case.dim, case.heads, case.lq
    e0 = _n(rng, (6, C), 0.1)
    x = _n(rng, (Lq, C), 1.0).to(torch.bfloat16).float()
    rows = list(case.lead_rows) if case.lead_rows else [Lq] * case.n_lead
    k_lead = [_n(rng, (r, H, HEAD_DIM), 1.0).to(torch.bfloat16) for r in rows]
    v_lead = [_n(rng, (r, H, HEAD_DIM), 1.0).to(torch.bfloat16) for r in rows]
    ctx = _n(rng, (case.text_len, C), 1.0).to(torch.bfloat16)
    if case.dedup_rows:
        ctx[case.dedup_rows:] = ctx[case.dedup_rows]
    film = None
    if case.film:
        film = (_n(rng, (Lq, C), 0.1).to(torch.bfloat16), _n(rng, (Lq, C), 0.1).to(torch.bfloat16))
    inp = dict(x=x, e0=e0, k_lead=k_lead, v_lead=v_lead, context=ctx, film=film)
    if case.cam:   # drawn after everything else, so the draws above are the same with or without it
        for nm in ("cam_injector_layer1", "cam_injector_layer2", "cam_scale_layer", "cam_shift_layer"):
            p[f"{nm}.weight"] = _n(rng, (C, C), 0.02).to(torch.bfloat16)
            p[f"{nm}.bias"] = _n(rng, (C,), 0.02).to(torch.bfloat16)
        inp["cam"] = _n(rng, (Lq, C), 1.0).to(torch.bfloat16)
    return p, inp


@dataclass
class ModelCase:
    """A whole causal-fast DiT forward (WanModelFast, model_fast.py:3151-3283) at a tiny i2v geometry."""
    dim: int = 256
    ffn: int = 256
    layers: int = 2
    in_dim: int = 36               # 16 latent channels + 20 image-condition channels (y)
    x_dim: int = 16
    out_dim: int = 16
    text_dim: int = 64
    text_len: int = 32
    ctx_rows: int = 20             # prompt rows before the zero padding to text_len
    freq_dim: int = 256
    latent: tuple = (3, 8, 12)     # (frames, H, W) of the chunk's latent; patch (1, 2, 2)
    n_chunks: int = 3
    chunk_index: int = 2           # which chunk of the rolling cache this forward writes
    timestep: float = 500.0
    seed: int = 11

    @property
    def heads(self):
        return self.dim // HEAD_DIM

    @property
    def grid(self):
        f, h, w = self.latent
        return f, h // 2, w // 2

    @property
    def lq(self):
        f, h, w = self.grid
        return f * h * w


def make_model_case(case: ModelCase):
    """Returns (state_dict, inputs) as CPU tensors. Linear / Conv3d weights and biases ~N(0, 0.02), block
    parameters as make_params (+ camera layers), modulations ~N(0, 0.1); x, y ~N(0, 1) fp32, the prompt and
    the camera condition ~N(0, 1) bf16, the leading cache chunks ~N(0, 1) bf16. Module dtypes follow the
    reference pipeline: bf16 weights except the timestep MLPs, the head and each block's modulation / norm3
    (fp32)."""
    rng = np.random.Generator(np.random.PCG64(case.seed))
    bf = torch.bfloat16
    C, T = case.dim, case.text_dim
    sd = {}
    sd["patch_embedding.weight"] = _n(rng, (C, case.in_dim, 1, 2, 2), 0.02).to(bf)
    sd["patch_embedding.bias"] = _n(rng, (C,), 0.02).to(bf)
    sd["patch_embedding_wancamctrl.weight"] = _n(rng, (C, 6 * 64 * 4), 0.02).to(bf)
    sd["patch_embedding_wancamctrl.bias"] = _n(rng, (C,), 0.02).to(bf)
    for nm in ("c2ws_hidden_states_layer1", "c2ws_hidden_states_layer2"):
        sd[f"{nm}.weight"] = _n(rng, (C, C), 0.02).to(bf)
        sd[f"{nm}.bias"] = _n(rng, (C,), 0.02).to(bf)
    sd["text_embedding.0.weight"] = _n(rng, (C, T), 0.02).to(bf)
    sd["text_embedding.0.bias"] = _n(rng, (C,), 0.02).to(bf)
    sd["text_embedding.2.weight"] = _n(rng, (C, C), 0.02).to(bf)
    sd["text_embedding.2.bias"] = _n(rng, (C,), 0.02).to(bf)
    sd["time_embedding.0.weight"] = _n(rng, (C, case.freq_dim), 0.02)
    sd["time_embedding.0.bias"] = _n(rng, (C,), 0.02)
    sd["time_embedding.2.weight"] = _n(rng, (C, C), 0.02)
    sd["time_embedding.2.bias"] = _n(rng, (C,), 0.02)
    sd["time_projection.1.weight"] = _n(rng, (6 * C, C), 0.02)
    sd["time_projection.1.bias"] = _n(rng, (6 * C,), 0.02)
    bcase = BlockCase(dim=C, ffn=case.ffn)
    for i in range(case.layers):
        p = make_params(bcase, rng)
        for nm in ("cam_injector_layer1", "cam_injector_layer2", "cam_scale_layer", "cam_shift_layer"):
            p[f"{nm}.weight"] = _n(rng, (C, C), 0.02).to(bf)
            p[f"{nm}.bias"] = _n(rng, (C,), 0.02).to(bf)
        for k, v in p.items():
            sd[f"blocks.{i}.{k}"] = v
    sd["head.head.weight"] = _n(rng, (case.out_dim * 4, C), 0.02)
    sd["head.head.bias"] = _n(rng, (case.out_dim * 4,), 0.02)
    sd["head.modulation"] = _n(rng, (1, 2, C), 0.1)
    f, h, w = case.latent
    x = _n(rng, (case.x_dim, f, h, w), 1.0)
    y = _n(rng, (case.in_dim - case.x_dim, f, h, w), 1.0)
    ctx = _n(rng, (case.ctx_rows, T), 1.0).to(bf)
    cam = _n(rng, (1, 6 * 64, f, h, w), 1.0).to(bf)
    lq, H = case.lq, case.heads
    lead = [[(_n(rng, (lq, H, HEAD_DIM), 1.0).to(bf), _n(rng, (lq, H, HEAD_DIM), 1.0).to(bf))
             for _ in range(case.n_chunks)] for _ in range(case.layers)]
    inp = dict(x=x, y=y, context=ctx, cam=cam, t=torch.tensor([case.timestep]), cache=lead)
    return sd, inp
