"""CPU restatement of one causal-fast WanModelFast.forward on the chunked KV cache.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows yahavb/lingbot-world-v2 wan/modules/model_fast.py, default (non-TP, single-rank, chunked cache,
hoisted camera FiLM) path, keeping the reference's dtypes:
  * patch embedding: Conv3d(in_dim, dim, k = s = (1, 2, 2)) on cat([x, y]) in bf16, tokens frame-major
    (:3384-3390, i2v concat :3356-3357)
  * text embedding: prompt zero-padded to text_len, Linear -> GELU(tanh) -> Linear in bf16 (:3456-3468)
  * timestep: sinusoidal_embedding_1d in fp64 (wan/modules/model.py:16-26) -> fp32 time_embedding MLP ->
    e [1, dim]; e0 = time_projection(e) [6, dim] (:3414-3446)
  * camera: '1 c (f c1) (h c2) (w c3) -> 1 (f h w) (c c1 c2 c3)' -> patch_embedding_wancamctrl ->
    emb + layer2(silu(layer1(emb))) (:3505-3552); per block cam_film on it (_cam_films :4242, hoisted)
  * RoPE grids at start_frame = current_start // frame_seqlen (:3652-3663); chunk_routing picks the
    destination and leading chunks (:3669-3673)
  * the blocks (oracle.block.block_forward) on the fp32 residual (:3771, :3830-3852)
  * CausalHead: LN(x) * (1 + e1) + e0 with e = modulation + e, fp32 Linear (:3119-3148); unpatchify (:4419-4440)
"""

import torch
import torch.nn.functional as F

from . import block as ob

HEAD_DIM = 128


def sinusoidal_embedding_1d(dim, position):
    """wan/modules/model.py:16-26: cos | sin of position * 10000^(-i/half), fp64."""
    half = dim // 2
    position = position.to(torch.float64)
    s = torch.outer(position, torch.pow(10000, -torch.arange(half).to(position).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


def patch_tokens(v, patch=(1, 2, 2)):
    """[C, F, H, W] -> [F/pt * H/ph * W/pw, C * pt * ph * pw], columns in Conv3d weight order (c, kt, kh, kw)."""
    c, f, h, w = v.shape
    pt, ph, pw = patch
    t = v.reshape(c, f // pt, pt, h // ph, ph, w // pw, pw)
    return t.permute(1, 3, 5, 0, 2, 4, 6).reshape((f // pt) * (h // ph) * (w // pw), c * pt * ph * pw)


def patch_embed(sd, x_cat):
    w = sd["patch_embedding.weight"]
    return ob.linear(patch_tokens(x_cat.to(torch.bfloat16)), w.reshape(w.shape[0], -1), sd["patch_embedding.bias"])


def text_embed(sd, ctx, text_len):
    c = torch.cat([ctx, ctx.new_zeros(text_len - ctx.shape[0], ctx.shape[1])]).to(torch.bfloat16)
    h = ob.linear(c, sd["text_embedding.0.weight"], sd["text_embedding.0.bias"])
    h = F.gelu(h.float(), approximate="tanh").to(torch.bfloat16)
    return ob.linear(h, sd["text_embedding.2.weight"], sd["text_embedding.2.bias"])


def time_embed(sd, t, freq_dim):
    s = sinusoidal_embedding_1d(freq_dim, t.flatten()).float()
    e = F.linear(s, sd["time_embedding.0.weight"].float(), sd["time_embedding.0.bias"].float())
    e = F.linear(F.silu(e), sd["time_embedding.2.weight"].float(), sd["time_embedding.2.bias"].float())
    e0 = F.linear(F.silu(e), sd["time_projection.1.weight"].float(), sd["time_projection.1.bias"].float())
    return e, e0.reshape(6, -1)


def camera_embed(sd, cam, patch=(1, 2, 2)):
    """cam [1, c, F, H, W] -> [L, dim] bf16."""
    c = patch_tokens(cam[0], patch).to(torch.bfloat16)
    emb = ob.linear(c, sd["patch_embedding_wancamctrl.weight"], sd["patch_embedding_wancamctrl.bias"])
    h = F.silu(ob.linear(emb, sd["c2ws_hidden_states_layer1.weight"], sd["c2ws_hidden_states_layer1.bias"]).float())
    h = ob.linear(h.to(torch.bfloat16), sd["c2ws_hidden_states_layer2.weight"], sd["c2ws_hidden_states_layer2.bias"])
    return (emb + h).to(torch.bfloat16)


def head(sd, x, e, eps=1e-6):
    m = (sd["head.modulation"].float().reshape(2, -1) + e.float().reshape(1, -1)).chunk(2, dim=0)
    h = ob.layer_norm(x.float(), eps) * (1 + m[1]) + m[0]
    return F.linear(h, sd["head.head.weight"].float(), sd["head.head.bias"].float())


def unpatchify(u, grid, out_dim, patch=(1, 2, 2)):
    f, h, w = grid
    u = u[: f * h * w].reshape(f, h, w, *patch, out_dim)
    u = torch.einsum("fhwpqrc->cfphqwr", u)
    return u.reshape(out_dim, *[a * b for a, b in zip(grid, patch)])


def block_params(sd, i):
    pre = f"blocks.{i}."
    return {k[len(pre):]: v for k, v in sd.items() if k.startswith(pre)}


def model_forward(sd, inp, case, chunk_routing, seq_len=None, rope_dtype=None):
    """Returns (out [out_dim, F, H, W] fp32, per-layer destination K and V, per-layer context K and V).
    seq_len is the forward's seq_len (default: the chunk's tokens); from 4,096 on the reference switches its RoPE to
    bf16 (model_fast.py:1144-1148, :3348), which rope_dtype overrides (the reference keeps bf16 for the rest of the
    process once any forward has switched it)."""
    x_cat = torch.cat([inp["x"], inp["y"]], dim=0)
    tokens = patch_embed(sd, x_cat).float()
    ctx = text_embed(sd, inp["context"], case.text_len)
    e, e0 = time_embed(sd, inp["t"], case.freq_dim)
    cam = camera_embed(sd, inp["cam"])
    grid = case.grid
    L = case.lq
    start_frame = (case.chunk_index * L) // (grid[1] * grid[2])
    cos, sin = ob.rope_grid(ob.rope_freqs(), grid, start_frame)
    if rope_dtype is None:
        rope_dtype = torch.bfloat16 if (L if seq_len is None else seq_len) >= 4096 else torch.float32
    dest, leading = chunk_routing(case.chunk_index, case.n_chunks)
    x = tokens
    k_dest, v_dest, ctx_k, ctx_v = [], [], [], []
    for i in range(case.layers):
        p = block_params(sd, i)
        film = ob.cam_film(p, cam)
        ck, cv = ob.cross_kv(p, ctx)
        lead = inp["cache"][i]
        k_lead = [lead[s][0] for s in leading]
        v_lead = [lead[s][1] for s in leading]
        r = ob.block_forward(p, x, e0, k_lead, v_lead, ck, cv, cos, sin, film=film, return_all=True,
                             rope_dtype=rope_dtype)
        x = r["x"]
        k_dest.append(r["k"].to(torch.bfloat16))
        v_dest.append(r["v"].to(torch.bfloat16))
        ctx_k.append(ck)
        ctx_v.append(cv)
    out = unpatchify(head(sd, x, e), grid, case.out_dim)
    return out, k_dest, v_dest, ctx_k, ctx_v
