"""CPU restatement of the Wan 2.1 VAE decoder (the frame path after the DiT) -- TEST INFRASTRUCTURE ONLY.

Follows yahavb/lingbot-world-v2 wan/modules/vae2_1.py in fp32 on CPU:
  * CausalConv3d (:16-35): zero padding of 2 * pad_t frames in front (none behind), spatial padding both sides;
    a cached tail of the previous call replaces that many front zeros
  * RMS_norm (:38-53): x / max(||x||_2 over channels, 1e-12) * sqrt(C) * gamma
  * Resample upsample2d / upsample3d (:65-158): nearest 2x in h, w, then Conv2d(C, C/2, 3, pad 1); upsample3d
    first runs the causal time_conv (C -> 2C, kernel (3, 1, 1)) and interleaves its two channel halves as frames
    2t, 2t + 1 -- except on the first call, whose frame is not time-upsampled ('Rep')
  * ResidualBlock (:185-219): RMS -> SiLU -> conv3x3x3 -> RMS -> SiLU -> conv3x3x3, plus the shortcut
    (1x1x1 conv when the width changes)
  * AttentionBlock (:222-267): per frame, RMS (2-D) -> 1x1 qkv -> single-head softmax attention over the h*w
    tokens -> 1x1 proj, plus the input
  * Decoder3d (:374-477) with its per-conv feature cache (the last CACHE_T = 2 input frames of every causal
    conv), called once per latent frame by WanVAE_.decode (:548-572) / decode_chunk (:574-596), after
    z * std + mean and the 1x1x1 conv2; Wan2_1_VAE.decode clamps to [-1, 1] (:685-691).
Parameters are a dict keyed by the reference's state-dict names (conv2.*, decoder.*).
"""
import math

import numpy as np
import torch
import torch.nn.functional as F

CACHE_T = 2


# ---------------------------------------------------------------------------------------------- structure
def decoder_layout(dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, temperal_upsample=(True, True, False)):
    """The decoder's module list as (kind, name, in_dim, out_dim) in forward order (Decoder3d.__init__ :376-426).
    kinds: conv (causal 3x3x3), res, attn, up3d, up2d, head."""
    dims = [dim * u for u in [dim_mult[-1]] + list(dim_mult[::-1])]
    mods = [("conv", "decoder.conv1", z_dim, dims[0]),
            ("res", "decoder.middle.0", dims[0], dims[0]),
            ("attn", "decoder.middle.1", dims[0], dims[0]),
            ("res", "decoder.middle.2", dims[0], dims[0])]
    idx = 0
    for i, (in_dim, out_dim) in enumerate(zip(dims[:-1], dims[1:])):
        if i in (1, 2, 3):
            in_dim = in_dim // 2
        for _ in range(num_res_blocks + 1):
            mods.append(("res", f"decoder.upsamples.{idx}", in_dim, out_dim))
            idx += 1
            in_dim = out_dim
        if i != len(dim_mult) - 1:
            mods.append(("up3d" if temperal_upsample[i] else "up2d", f"decoder.upsamples.{idx}", out_dim, out_dim // 2))
            idx += 1
    mods.append(("head", "decoder.head", dims[-1], 3))
    return mods


def param_shapes(dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, temperal_upsample=(True, True, False)):
    """State-dict names and shapes of conv2 + the decoder, in a fixed order."""
    out = [("conv2.weight", (z_dim, z_dim, 1, 1, 1)), ("conv2.bias", (z_dim,))]
    for kind, name, ci, co in decoder_layout(dim, z_dim, dim_mult, num_res_blocks, temperal_upsample):
        if kind == "conv":
            out += [(f"{name}.weight", (co, ci, 3, 3, 3)), (f"{name}.bias", (co,))]
        elif kind == "res":
            out += [(f"{name}.residual.0.gamma", (ci, 1, 1, 1)),
                    (f"{name}.residual.2.weight", (co, ci, 3, 3, 3)), (f"{name}.residual.2.bias", (co,)),
                    (f"{name}.residual.3.gamma", (co, 1, 1, 1)),
                    (f"{name}.residual.6.weight", (co, co, 3, 3, 3)), (f"{name}.residual.6.bias", (co,))]
            if ci != co:
                out += [(f"{name}.shortcut.weight", (co, ci, 1, 1, 1)), (f"{name}.shortcut.bias", (co,))]
        elif kind == "attn":
            out += [(f"{name}.norm.gamma", (ci, 1, 1)), (f"{name}.to_qkv.weight", (3 * ci, ci, 1, 1)),
                    (f"{name}.to_qkv.bias", (3 * ci,)), (f"{name}.proj.weight", (ci, ci, 1, 1)),
                    (f"{name}.proj.bias", (ci,))]
        elif kind in ("up3d", "up2d"):
            out += [(f"{name}.resample.1.weight", (ci // 2, ci, 3, 3)), (f"{name}.resample.1.bias", (ci // 2,))]
            if kind == "up3d":
                out += [(f"{name}.time_conv.weight", (2 * ci, ci, 3, 1, 1)), (f"{name}.time_conv.bias", (2 * ci,))]
        elif kind == "head":
            out += [(f"{name}.0.gamma", (ci, 1, 1, 1)), (f"{name}.2.weight", (3, ci, 3, 3, 3)),
                    (f"{name}.2.bias", (3,))]
    return out


def make_params(seed=0, **cfg):
    """Seeded fp32 parameters: conv weights ~N(0, 1 / fan_in), biases ~N(0, 0.02), RMS gammas 1 + N(0, 0.1)
    (the reference zero-initialises proj; random here so that the attention path is exercised)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    p = {}
    for name, shape in param_shapes(**cfg):
        if name.endswith("gamma"):
            v = 1.0 + 0.1 * rng.standard_normal(shape)
        elif name.endswith("bias"):
            v = 0.02 * rng.standard_normal(shape)
        else:
            fan_in = int(np.prod(shape[1:]))
            v = rng.standard_normal(shape) / math.sqrt(fan_in)
        p[name] = torch.from_numpy(v.astype(np.float32))
    return p


# ---------------------------------------------------------------------------------------------- ops
def causal_conv3d(x, w, b, cache=None):
    """x [1, C, T, H, W]; w [Co, C, kt, kh, kw]; 2 * (kt // 2) front frames: the cache tail, then zeros."""
    kt, kh, kw = w.shape[2:]
    pt = 2 * (kt // 2)
    if pt and cache is not None:
        x = torch.cat([cache, x], dim=2)
        pt -= cache.shape[2]
    x = F.pad(x, (kw // 2, kw // 2, kh // 2, kh // 2, pt, 0))
    return F.conv3d(x, w, b)


def rms_norm(x, gamma):
    """F.normalize over the channel dim (eps 1e-12) * sqrt(C) * gamma."""
    c = x.shape[1]
    return x / x.norm(dim=1, keepdim=True).clamp_min(1e-12) * math.sqrt(c) * gamma.view(1, c, *([1] * (x.dim() - 2)))


def _tail(x, prev):
    """The last CACHE_T frames of the layer input, reaching into the previous cache when x is shorter."""
    t = x[:, :, -CACHE_T:]
    if t.shape[2] < CACHE_T and prev is not None:
        t = torch.cat([prev[:, :, -1:], t], dim=2)
    return t


class Decoder:
    """Decoder3d + the per-conv cache of one decode (WanVAE_._feat_map)."""

    def __init__(self, params, **cfg):
        self.p = params
        self.layout = decoder_layout(**cfg)
        self.cache = {}

    def _conv(self, key, x, w, b):
        prev = self.cache.get(key)
        out = causal_conv3d(x, w, b, prev)
        self.cache[key] = _tail(x, prev)
        return out

    def _res(self, name, x):
        p = self.p
        h = x
        if f"{name}.shortcut.weight" in p:
            h = F.conv3d(x, p[f"{name}.shortcut.weight"], p[f"{name}.shortcut.bias"])
        y = F.silu(rms_norm(x, p[f"{name}.residual.0.gamma"]))
        y = self._conv(f"{name}.residual.2", y, p[f"{name}.residual.2.weight"], p[f"{name}.residual.2.bias"])
        y = F.silu(rms_norm(y, p[f"{name}.residual.3.gamma"]))
        y = self._conv(f"{name}.residual.6", y, p[f"{name}.residual.6.weight"], p[f"{name}.residual.6.bias"])
        return y + h

    def _attn(self, name, x):
        p = self.p
        _, c, t, h, w = x.shape
        frames = x[0].permute(1, 0, 2, 3)                           # [t, c, h, w]
        y = rms_norm(frames, p[f"{name}.norm.gamma"])
        qkv = F.conv2d(y, p[f"{name}.to_qkv.weight"], p[f"{name}.to_qkv.bias"])
        qkv = qkv.reshape(t, 3 * c, h * w).permute(0, 2, 1)        # [t, hw, 3c]
        q, k, v = qkv.chunk(3, dim=-1)
        a = torch.softmax(q @ k.transpose(1, 2) / math.sqrt(c), dim=-1) @ v
        a = a.permute(0, 2, 1).reshape(t, c, h, w)
        out = F.conv2d(a, p[f"{name}.proj.weight"], p[f"{name}.proj.bias"])
        return x + out.permute(1, 0, 2, 3).unsqueeze(0)

    def _resample(self, kind, name, x):
        p = self.p
        _, c, t, h, w = x.shape
        if kind == "up3d":
            key = f"{name}.time_conv"
            if key not in self.cache:
                self.cache[key] = "Rep"                              # first call: no temporal upsampling
            else:
                prev = self.cache[key]
                tail = x[:, :, -CACHE_T:]
                if tail.shape[2] < CACHE_T:
                    lead = torch.zeros_like(tail) if prev == "Rep" else prev[:, :, -1:]
                    tail = torch.cat([lead, tail], dim=2)
                y = causal_conv3d(x, p[f"{key}.weight"], p[f"{key}.bias"], None if prev == "Rep" else prev)
                self.cache[key] = tail
                y = y.reshape(1, 2, c, t, h, w)
                x = torch.stack((y[:, 0], y[:, 1]), dim=3).reshape(1, c, 2 * t, h, w)
        t = x.shape[2]
        frames = x[0].permute(1, 0, 2, 3)
        frames = F.interpolate(frames, scale_factor=(2.0, 2.0), mode="nearest-exact")
        frames = F.conv2d(frames, p[f"{name}.resample.1.weight"], p[f"{name}.resample.1.bias"], padding=1)
        return frames.permute(1, 0, 2, 3).unsqueeze(0)

    def frame(self, x):
        """One Decoder3d call on x [1, z, 1, h, w] (one latent frame)."""
        p = self.p
        for kind, name, _, _ in self.layout:
            if kind == "conv":
                x = self._conv(name, x, p[f"{name}.weight"], p[f"{name}.bias"])
            elif kind == "res":
                x = self._res(name, x)
            elif kind == "attn":
                x = self._attn(name, x)
            elif kind in ("up3d", "up2d"):
                x = self._resample(kind, name, x)
            else:
                x = F.silu(rms_norm(x, p[f"{name}.0.gamma"]))
                x = self._conv(f"{name}.2", x, p[f"{name}.2.weight"], p[f"{name}.2.bias"])
        return x


# Wan2_1_VAE latent statistics (vae2_1.py:656-665), held in bf16 there; scale = [mean, 1 / std] (:666-667)
LATENT_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508,
               0.4134, -0.0715, 0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921]
LATENT_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743,
              3.2687, 2.1526, 2.8652, 1.5579, 1.6382, 1.1253, 2.8251, 1.9160]


def latent_scale(dtype=torch.bfloat16):
    mean = torch.tensor(LATENT_MEAN, dtype=dtype)
    std = torch.tensor(LATENT_STD, dtype=dtype)
    return [mean, 1.0 / std]


def decode(params, z, scale=None, decoder=None, **cfg):
    """z [z_dim, T, h, w] -> video [3, T', 8h, 8w] in [-1, 1] (Wan2_1_VAE.decode / decode_chunk with a
    decoder carried across calls); z / scale[1] + scale[0] as WanVAE_.decode does (:555-559)."""
    dec = decoder if decoder is not None else Decoder(params, **cfg)
    scale = scale if scale is not None else latent_scale()
    zc = z.unsqueeze(0) / scale[1].view(1, -1, 1, 1, 1) + scale[0].view(1, -1, 1, 1, 1)
    x = F.conv3d(zc, params["conv2.weight"], params["conv2.bias"])
    out = torch.cat([dec.frame(x[:, :, i:i + 1]) for i in range(x.shape[2])], dim=2)
    return out.clamp(-1, 1)[0], dec
