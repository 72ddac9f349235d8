"""CPU restatement of CausalWanAttentionBlock.forward (non-TP, chunked-KV path).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows yahavb/lingbot-world-v2 wan/modules/model_fast.py with the plain-PyTorch fallbacks the
block takes off-Neuron, keeping the reference's rounding points:
  * adaLN: e = modulation + e0 in fp32, chunked in 6 (model_fast.py:2954-2955)
  * h = LN(x) * (1 + e1) + e0 in fp32 (:3045; WanLayerNorm model.py:145-156), cast to bf16 in qkv_fn (:1733)
  * q/k/v = bf16 nn.Linear; q, k = WanRMSNorm (model.py:134-143: fp32 norm, type_as(bf16), * bf16 weight)
  * RoPE: precomputed cos/sin grids (model_fast.py:878-931) applied in fp32, .type_as(v) (:933-979, :1893-1900)
  * chunked cache: the new chunk's roped K and V are the destination chunk (LAST), attention over
    (leading..., destination) with no mask (:2398-2418, attention.py:1048-1058, SDPA :1134-1143)
  * o-projection (:2709-2750); x = x + y * e2 in fp32 (:3063-3065); hoisted camera FiLM
    x = (1 + cam_scale) * x + cam_shift with bf16 FiLM tensors (:3056-3089)
  * cross-attention on norm3(x) (affine LN) with cached context K/V (:2755-2834), optional
    cross_dedup (attention.py:516-554)
  * h = (LN(x) * (1 + e4) + e3).to(bf16) (:3101); FFN Linear -> GELU(tanh) -> Linear (:2870-2872) or the
    MXFP8 FFN (_ffn_mx :1584-1611) emulated with oracle.mx; x = x + y * e5 (:3110-3111).
  * LINGBOT_LIN_MX (:1266-1269, :1442-1494): the Linears named in mx_linears (q/k/v/o of both attentions, the
    camera-FiLM MLP) become _mx_matmul (:1403-1410): bf16(mm(x, W)) + b in bf16, emulated with oracle.mx.
"""
import math

import torch
import torch.nn.functional as F

from . import mx as mxo

HEAD_DIM = 128


# --------------------------------------------------------------------------------------------
# RoPE tables: wan/modules/model.py:47-53 (rope_params), model_fast.py:3273-3278 (freqs concat),
# model_fast.py:878-931 (_causal_rope_grids_build)
# --------------------------------------------------------------------------------------------
def rope_params(max_seq_len, dim, theta=10000):
    return torch.outer(torch.arange(max_seq_len).float(),
                       1.0 / torch.pow(theta, torch.arange(0, dim, 2).float().div(dim)))


def rope_freqs(head_dim=HEAD_DIM, max_frames=1024):
    d = head_dim
    return torch.cat([rope_params(max_frames, d - 4 * (d // 6)),
                      rope_params(max_frames, 2 * (d // 6)),
                      rope_params(max_frames, 2 * (d // 6))], dim=1)


def rope_split(freqs):
    c = freqs.shape[1]
    s0, s1 = c - 2 * (c // 3), c // 3
    return s0, s1


def rope_grid(freqs, grid, start_frame):
    """cos, sin [f*h*w, c] (fp32) for the full frame-major grid of one chunk."""
    f, h, w = grid
    c = freqs.shape[1]
    s0, s1 = rope_split(freqs)
    fs = freqs.split([s0, s1, s1], dim=1)
    ang = torch.cat([fs[0][start_frame:start_frame + f].view(f, 1, 1, -1).expand(f, h, w, -1),
                     fs[1][:h].view(1, h, 1, -1).expand(f, h, w, -1),
                     fs[2][:w].view(1, 1, w, -1).expand(f, h, w, -1)], dim=-1).reshape(f * h * w, c)
    return torch.cos(ang), torch.sin(ang)


def rope_apply(x, cos, sin, dtype=torch.float32):
    """x [L, H, d] bf16 -> rotated bf16 (interleaved (re, im) pairs), model_fast.py:933-979. dtype is the
    reference's RoPE dtype (ROPE_DTYPE, :985-1003): fp32 math by default; bf16 once a model forward has seen a
    chunk of 4,096 or more tokens (:1144-1148), when the grids are cast to bf16 (:928-929) and every product and sum
    of the rotation is a bf16 op."""
    L, H, d = x.shape
    xf = x.to(dtype).reshape(L, H, d // 2, 2)
    re, im = xf[..., 0], xf[..., 1]
    c, s = cos.to(dtype).view(L, 1, -1), sin.to(dtype).view(L, 1, -1)
    out = torch.stack([re * c - im * s, re * s + im * c], dim=-1)
    return out.reshape(L, H, d).to(x.dtype)


# --------------------------------------------------------------------------------------------
# primitives
# --------------------------------------------------------------------------------------------
def linear(x, w, b):
    """bf16 nn.Linear: fp32 accumulation, one rounding to bf16."""
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    return y.to(torch.bfloat16)


def mx_matmul(x, w, b, fmt="e4m3"):
    """_mx_matmul (model_fast.py:1403-1410): the MXFP8 matmul's bf16 result, then + bias in bf16; fmt is the element
    format LINGBOT_MX_FP8 selects (kernels/ffn_mx.py:8,18)."""
    y = mxo.mx_linear(x.to(torch.bfloat16), w, fmt)
    return y if b is None else (y.float() + b.float()).to(torch.bfloat16)


def block_linear(p, name, x, mx_linears=(), fmt="e4m3"):
    """Block Linear `name` (e.g. "self_attn.q") on x: nn.Linear, or _mx_matmul when LINGBOT_LIN_MX quantises it (in
    the element format fmt of LINGBOT_MX_FP8)."""
    w, b = p[name + ".weight"], p.get(name + ".bias")
    return mx_matmul(x, w, b, fmt) if name in mx_linears else linear(x, w, b)


def rms_norm(x, weight, eps):
    """WanRMSNorm: fp32 normalisation, cast back to x's dtype, times the (bf16) weight."""
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)).to(x.dtype)
    return n * weight


def layer_norm(x, eps, weight=None, bias=None):
    return F.layer_norm(x.float(), (x.shape[-1],), weight, bias, eps)


def attention(q, k, v, key_bias=None, head_block=4):
    """softmax(q kᵀ / sqrt(d) + bias) v, fp32 math -> bf16. q [Lq, H, d], k/v [Lk, H, d]."""
    Lq, H, d = q.shape
    out = torch.empty(Lq, H, d, dtype=torch.float32)
    scale = 1.0 / math.sqrt(d)
    for h0 in range(0, H, head_block):
        qh = q[:, h0:h0 + head_block].float().permute(1, 0, 2)
        kh = k[:, h0:h0 + head_block].float().permute(1, 2, 0)
        vh = v[:, h0:h0 + head_block].float().permute(1, 0, 2)
        s = torch.matmul(qh, kh) * scale
        if key_bias is not None:
            s = s + key_bias.float().view(1, 1, -1)
        p = torch.softmax(s, dim=-1)
        out[:, h0:h0 + head_block] = torch.matmul(p, vh).permute(1, 0, 2)
    return out.to(torch.bfloat16)


def cross_dedup_bias(k, v, kc):
    """attention.py:516-523: log(m / r) on the r rows among the first kc that equal the last row
    of both K and V (m such rows overall), 0 elsewhere. k, v [L, H, d]."""
    same = (k == k[-1:]).flatten(1).all(dim=1) & (v == v[-1:]).flatten(1).all(dim=1)
    s = same[:kc]
    m, r = same.sum().float(), s.sum().float()
    return torch.where(s, torch.log(m / r), torch.zeros((), dtype=torch.float32))


# --------------------------------------------------------------------------------------------
# block
# --------------------------------------------------------------------------------------------
def cross_kv(p, context, eps=1e-6, mx_linears=(), mx_fmt="e4m3"):
    """Cross-attention K/V of the text context, filled on the first call (model_fast.py:2784-2798)."""
    C = context.shape[-1]
    H = C // HEAD_DIM
    ctx = context.reshape(-1, C).to(torch.bfloat16)
    k = rms_norm(block_linear(p, "cross_attn.k", ctx, mx_linears, mx_fmt), p["cross_attn.norm_k.weight"], eps)
    v = block_linear(p, "cross_attn.v", ctx, mx_linears, mx_fmt)
    return k.view(-1, H, HEAD_DIM), v.view(-1, H, HEAD_DIM)


def block_forward(p, x, e0, k_lead, v_lead, ctx_k, ctx_v, cos, sin, film=None, mx=False, eps=1e-6,
                  dedup_kc=None, return_all=False, mx_linears=(), mx_fmt="e4m3", rope_dtype=torch.float32):
    """One block. x [Lq, C] fp32; e0 [6, C] fp32; k_lead/v_lead lists of [L_i, H, d] bf16;
    ctx_k/ctx_v [T, H, d] bf16; cos/sin [Lq, 64] fp32; film = (scale, shift) [Lq, C] bf16; mx: MXFP8 FFN;
    mx_linears: names of the other Linears in MXFP8 (LINGBOT_LIN_MX); mx_fmt: the element format of every MX
    matmul ("e4m3", or "e5m2" for LINGBOT_MX_FP8=float8_e5m2, kernels/ffn_mx.py:8,18); rope_dtype: the rotation's
    arithmetic (rope_apply).
    Returns x_out (and, with return_all, the intermediates)."""
    lin = lambda name, t: block_linear(p, name, t, mx_linears, mx_fmt)  # noqa: E731
    Lq, C = x.shape
    H = C // HEAD_DIM
    e = (p["modulation"].reshape(6, C).float() + e0.float()).chunk(6, dim=0)
    e = [t.reshape(C) for t in e]

    # self-attention
    h = (layer_norm(x, eps) * (1 + e[1]) + e[0]).to(torch.bfloat16)
    q = rms_norm(lin("self_attn.q", h), p["self_attn.norm_q.weight"], eps)
    k = rms_norm(lin("self_attn.k", h), p["self_attn.norm_k.weight"], eps)
    v = lin("self_attn.v", h).view(Lq, H, HEAD_DIM)
    q = rope_apply(q.view(Lq, H, HEAD_DIM), cos, sin, rope_dtype)
    k = rope_apply(k.view(Lq, H, HEAD_DIM), cos, sin, rope_dtype)
    ks = torch.cat(list(k_lead) + [k], dim=0)
    vs = torch.cat(list(v_lead) + [v], dim=0)
    attn = attention(q, ks, vs)
    y = lin("self_attn.o", attn.reshape(Lq, C))
    x1 = x + y.float() * e[2]
    if film is not None:
        x1 = (1.0 + film[0]) * x1 + film[1]

    # cross-attention
    h3 = layer_norm(x1, eps, p["norm3.weight"].float(), p["norm3.bias"].float()).to(torch.bfloat16)
    qc = rms_norm(lin("cross_attn.q", h3), p["cross_attn.norm_q.weight"], eps)
    qc = qc.view(Lq, H, HEAD_DIM)
    if dedup_kc is not None:
        bias = cross_dedup_bias(ctx_k, ctx_v, dedup_kc)
        ca = attention(qc, ctx_k[:dedup_kc], ctx_v[:dedup_kc], key_bias=bias)
    else:
        ca = attention(qc, ctx_k, ctx_v)
    x2 = x1 + lin("cross_attn.o", ca.reshape(Lq, C)).float()

    # FFN
    h2 = (layer_norm(x2, eps) * (1 + e[4]) + e[3]).to(torch.bfloat16)
    if mx or mx_linears:
        u = mx_matmul(h2, p["ffn.0.weight"], p["ffn.0.bias"], mx_fmt)
        g = F.gelu(u.float(), approximate="tanh").to(torch.bfloat16)
        y2 = mx_matmul(g, p["ffn.2.weight"], p["ffn.2.bias"], mx_fmt)
    else:
        u = linear(h2, p["ffn.0.weight"], p["ffn.0.bias"])
        g = F.gelu(u.float(), approximate="tanh").to(torch.bfloat16)
        y2 = linear(g, p["ffn.2.weight"], p["ffn.2.bias"])
    x3 = x2 + y2.float() * e[5]
    if return_all:
        return dict(x=x3, q=q, k=k, v=v, attn=attn, x1=x1, h3=h3, qc=qc, ca=ca, x2=x2, h2=h2, g=g, y2=y2)
    return x3


def cam_film(p, c, mx_linears=(), mx_fmt="e4m3"):
    """CausalWanAttentionBlock.cam_film (model_fast.py:2882-2891): bf16 Linears (or _mx_matmul under
    LINGBOT_LIN_MX), SiLU on the bf16 hidden, the camera embedding added to layer 2's bf16 output.
    c [L, C] bf16 -> (scale, shift) bf16."""
    lin = lambda name, t: block_linear(p, name, t, mx_linears, mx_fmt)  # noqa: E731
    h = F.silu(lin("cam_injector_layer1", c).float()).to(torch.bfloat16)
    h2 = (lin("cam_injector_layer2", h) + c).to(torch.bfloat16)
    return lin("cam_scale_layer", h2), lin("cam_shift_layer", h2)
