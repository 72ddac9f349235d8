"""Wan 2.1 VAE decoder on B200 (the frame path after the DiT: wan/modules/vae2_1.py).

Same decoder structure, state-dict names (conv2.*, decoder.*) and call semantics as the reference's WanVAE_
decode / decode_chunk (:548-596) and Wan2_1_VAE.decode / decode_chunk (:647-700): one Decoder3d pass per latent
frame, every causal convolution continuing from the last two input frames of the previous pass (the reference's
feature cache), the first frame not time-upsampled ('Rep', :100-135).

Layout: activations are frames stored channels-last with a one-pixel zero border, [frames][h + 2][w + 2][C]
bf16, C rounded up to a multiple of 32 (the 96-channel full-resolution level is stored at 96). Every causal
convolution (3x3x3, the (3,1,1) time_conv,
the 3x3 Resample conv, the 1x1x1 shortcut) is one implicit-GEMM launch of the tcgen05 GEMM (lbw_vae_conv): the
kernel taps are constant row shifts of that layout, the two history frames sit in front of the current ones in
a per-layer buffer, and the epilogue adds the bias and the shortcut and zeroes the border. RMS_norm + SiLU,
the nearest 2x upsampling and the time interleave are HBM-bound row kernels; the mid-block attention runs its
scores, probabilities and output through the GEMMs (fp32 scores, bf16 probabilities).
"""
import math

import torch
import torch.nn as nn

from . import kernels

BF16 = torch.bfloat16
CACHE_T = 2
# Wan2_1_VAE latent statistics (vae2_1.py:656-665, held in bf16 there); decode uses scale = [mean, 1 / std]
LATENT_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508,
               0.4134, -0.0715, 0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921]
LATENT_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743,
              3.2687, 2.1526, 2.8652, 1.5579, 1.6382, 1.1253, 2.8251, 1.9160]


def _pad64(c):
    return (c + 63) // 64 * 64


def _pad32(c):
    """Stored channels of an activation: outputs are written in 32-column chunks."""
    return (c + 31) // 32 * 32


def decoder_layout(dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, temperal_upsample=(True, True, False)):
    """(kind, name, in_dim, out_dim) of Decoder3d's modules in forward order (vae2_1.py:376-426)."""
    dims = [dim * u for u in [dim_mult[-1]] + list(dim_mult[::-1])]
    mods = [("conv", "decoder.conv1", z_dim, dims[0]), ("res", "decoder.middle.0", dims[0], dims[0]),
            ("attn", "decoder.middle.1", dims[0], dims[0]), ("res", "decoder.middle.2", dims[0], dims[0])]
    idx = 0
    for i, (in_dim, out_dim) in enumerate(zip(dims[:-1], dims[1:])):
        if i in (1, 2, 3):
            in_dim = in_dim // 2
        for _ in range(num_res_blocks + 1):
            mods.append(("res", f"decoder.upsamples.{idx}", in_dim, out_dim))
            idx += 1
            in_dim = out_dim
        if i != len(dim_mult) - 1:
            mods.append(("up3d" if temperal_upsample[i] else "up2d", f"decoder.upsamples.{idx}", out_dim,
                         out_dim // 2))
            idx += 1
    mods.append(("head", "decoder.head", dims[-1], 3))
    return mods


def _param_shapes(layout, z_dim):
    out = [("conv2.weight", (z_dim, z_dim, 1, 1, 1)), ("conv2.bias", (z_dim,))]
    for kind, name, ci, co in layout:
        if kind == "conv":
            out += [(f"{name}.weight", (co, ci, 3, 3, 3)), (f"{name}.bias", (co,))]
        elif kind == "res":
            out += [(f"{name}.residual.0.gamma", (ci, 1, 1, 1)), (f"{name}.residual.2.weight", (co, ci, 3, 3, 3)),
                    (f"{name}.residual.2.bias", (co,)), (f"{name}.residual.3.gamma", (co, 1, 1, 1)),
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
        else:
            out += [(f"{name}.0.gamma", (ci, 1, 1, 1)), (f"{name}.2.weight", (3, ci, 3, 3, 3)),
                    (f"{name}.2.bias", (3,))]
    return out


class _Node(nn.Module):
    """Parameter container so that dotted reference names resolve as module paths."""


class _Hist:
    """Per-layer causal buffer: frames 0-1 hold the last two frames of the layer's input series (zeros before the
    first), frames 2.. the current call's input, written in place by the producer."""

    def __init__(self, P, c, tmax, device):
        self.P, self.c = P, c
        self.buf = torch.zeros((CACHE_T + tmax) * P, c, dtype=BF16, device=device)

    def slot(self, t):
        return self.buf[CACHE_T * self.P:(CACHE_T + t) * self.P]

    def rows(self, t):
        return (CACHE_T + t) * self.P

    def advance(self, t):
        """The series' last two frames -> frames 0-1 (frame by frame in increasing order: no overlap)."""
        P = self.P
        for i in range(CACHE_T):
            self.buf[i * P:(i + 1) * P].copy_(self.buf[(t + i) * P:(t + i + 1) * P])


class _Act:
    """Padded frames of one level: data [t * (h + 2) * (w + 2), cp] bf16."""

    def __init__(self, data, t, h, w, c):
        self.data, self.t, self.h, self.w, self.c = data, t, h, w, c

    @property
    def P(self):
        return (self.h + 2) * (self.w + 2)

    @property
    def cp(self):
        return self.data.shape[1]


class WanVAEDecoder(nn.Module):
    """conv2 + Decoder3d of WanVAE_ (reference parameter names) with the B200 kernels."""

    def __init__(self, dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2,
                 temperal_upsample=(True, True, False)):
        super().__init__()
        self.dim, self.z_dim = dim, z_dim
        self.layout = decoder_layout(dim, z_dim, dim_mult, num_res_blocks, temperal_upsample)
        for name, shape in _param_shapes(self.layout, z_dim):
            *path, leaf = name.split(".")
            mod = self
            for p in path:
                if not hasattr(mod, p):
                    mod.add_module(p, _Node())
                mod = getattr(mod, p)
            mod.register_parameter(leaf, nn.Parameter(torch.zeros(shape), requires_grad=False))
        self._packed = None
        self.clear_cache()

    # ------------------------------------------------------------------ weights
    @torch.no_grad()
    def prepare(self):
        """Pack every convolution as a [c_out_p, taps * c_k] bf16 matrix (K ordered kt, kh, kw, c; c_k = the stored
        input channels rounded up to 64, zero weights past them), biases as bf16 [c_out_p], RMS gammas as fp32
        [c_p] (c_p, c_out_p: channels rounded up to 32; zero padding everywhere)."""
        sd = dict(self.named_parameters())
        dev = sd["conv2.weight"].device
        if dev.type != "cuda":
            raise ValueError("move the VAE decoder to a CUDA device first")

        def conv(wname, bname, cout_p=None, halves=False):
            w = sd[wname].float()
            if w.dim() == 4:
                w = w.unsqueeze(2)                            # Conv2d -> kt = 1
            co, ci = w.shape[:2]
            cip = _pad64(_pad32(ci))
            if halves:                                        # time_conv: [c | c] -> [c_p | c_p]
                c = co // 2
                cp = _pad32(c)
                wp = torch.zeros(2 * cp, cip, *w.shape[2:], device=dev)
                wp[:c, :ci], wp[cp:cp + c, :ci] = w[:c], w[c:]
                bp = torch.zeros(2 * cp, device=dev)
                bp[:c], bp[cp:cp + c] = sd[bname][:c].float(), sd[bname][c:].float()
            else:
                cop = cout_p or _pad32(co)
                wp = torch.zeros(cop, cip, *w.shape[2:], device=dev)
                wp[:co, :ci] = w
                bp = torch.zeros(cop, device=dev)
                bp[:co] = sd[bname].float()
            wk = wp.permute(0, 2, 3, 4, 1).reshape(wp.shape[0], -1).to(BF16).contiguous()
            return wk, bp.to(BF16).contiguous(), tuple(w.shape[2:])

        def gamma(name):
            g = sd[name].float().reshape(-1)
            out = torch.zeros(_pad32(g.numel()), device=dev)
            out[:g.numel()] = g
            return out

        pk = {"conv2": conv("conv2.weight", "conv2.bias")}
        for kind, name, ci, co in self.layout:
            if kind == "conv":
                pk[name] = conv(f"{name}.weight", f"{name}.bias")
            elif kind == "res":
                pk[f"{name}.g0"] = gamma(f"{name}.residual.0.gamma")
                pk[f"{name}.c0"] = conv(f"{name}.residual.2.weight", f"{name}.residual.2.bias")
                pk[f"{name}.g1"] = gamma(f"{name}.residual.3.gamma")
                pk[f"{name}.c1"] = conv(f"{name}.residual.6.weight", f"{name}.residual.6.bias")
                if ci != co:
                    pk[f"{name}.sc"] = conv(f"{name}.shortcut.weight", f"{name}.shortcut.bias")
            elif kind == "attn":
                c, cp = ci, _pad64(ci)      # a GEMM operand: K = cp must be a multiple of 64
                if cp != _pad32(ci):
                    raise ValueError(f"the mid-block attention width {ci} must be a multiple of 64")
                g = gamma(f"{name}.norm.gamma")
                wq = sd[f"{name}.to_qkv.weight"].float().reshape(3 * c, c)
                bq = sd[f"{name}.to_qkv.bias"].float()
                w3 = torch.zeros(3 * cp, cp, device=dev)
                b3 = torch.zeros(3 * cp, device=dev)
                for j in range(3):
                    w3[j * cp:j * cp + c, :c] = wq[j * c:(j + 1) * c]
                    b3[j * cp:j * cp + c] = bq[j * c:(j + 1) * c]
                wo = torch.zeros(cp, cp, device=dev)
                wo[:c, :c] = sd[f"{name}.proj.weight"].float().reshape(c, c)
                bo = torch.zeros(cp, device=dev)
                bo[:c] = sd[f"{name}.proj.bias"].float()
                pk[name] = dict(g=g, wqkv=w3.to(BF16).contiguous(), bqkv=b3.to(BF16).contiguous(),
                                wo=wo.to(BF16).contiguous(), bo=bo.to(BF16).contiguous())
            elif kind in ("up3d", "up2d"):
                pk[f"{name}.rs"] = conv(f"{name}.resample.1.weight", f"{name}.resample.1.bias")
                if kind == "up3d":
                    pk[f"{name}.tc"] = conv(f"{name}.time_conv.weight", f"{name}.time_conv.bias", halves=True)
            else:
                pk[f"{name}.g"] = gamma(f"{name}.0.gamma")
                pk[f"{name}.c"] = conv(f"{name}.2.weight", f"{name}.2.bias", cout_p=32)
        self._packed = pk
        return pk

    def clear_cache(self):
        """WanVAE_.clear_cache (:610-617): a new video starts with zero history and the 'Rep' first frame."""
        self._hist = {}
        self._rep = set()

    # ------------------------------------------------------------------ layers
    def _hist_for(self, key, act, c_in_p, tmax):
        h = self._hist.get(key)
        if h is None or h.P != act.P or h.c != c_in_p:
            h = self._hist[key] = _Hist(act.P, c_in_p, tmax, act.data.device)
        return h

    def _conv_causal(self, key, act, producer, tmax, residual=None):
        """producer(dest) writes the layer input for act.t frames into the history buffer (None: already written
        there); then the causal convolution."""
        wk, bk, ks = self._packed[key]
        hist = self._hist_for(key, act, act.cp, tmax)
        if producer is not None:
            producer(hist.slot(act.t))
        out = torch.empty(act.t * act.P, wk.shape[0], dtype=BF16, device=act.data.device)
        kernels.vae_conv(hist.buf, hist.rows(act.t), act.cp, wk, bk, wk.shape[0], ks, act.t, act.h, act.w, out,
                         residual=residual)
        hist.advance(act.t)
        return out

    def _conv_plain(self, key, data, t, h, w, residual=None):
        wk, bk, ks = self._packed[key]
        out = torch.empty(t * (h + 2) * (w + 2), wk.shape[0], dtype=BF16, device=data.device)
        kernels.vae_conv(data, data.shape[0], data.shape[1], wk, bk, wk.shape[0], ks, t, h, w, out, residual=residual)
        return out

    def _rms(self, src, gamma, c_real, silu):
        def write(dest):
            kernels.vae_rms_silu(src, dest.shape[0], src.shape[1], c_real, gamma, silu, dest)
        return write

    def _res(self, name, ci, co, x, tmax):
        pk = self._packed
        h = self._conv_plain(f"{name}.sc", x.data, x.t, x.h, x.w) if ci != co else x.data
        wa, ba, ka = pk[f"{name}.c0"]
        cop = wa.shape[0]
        if cop <= 256:
            # the first convolution writes RMS + SiLU of its rows straight into the second one's input
            ha = self._hist_for(f"{name}.c0", x, x.cp, tmax)
            self._rms(x.data, pk[f"{name}.g0"], ci, True)(ha.slot(x.t))
            ya = _Act(x.data, x.t, x.h, x.w, co)                         # (shape only: P, device)
            hb = self._hist_for(f"{name}.c1", ya, cop, tmax)
            kernels.vae_conv_rms(ha.buf, ha.rows(x.t), x.cp, wa, ba, cop, ka, x.t, x.h, x.w, pk[f"{name}.g1"], co,
                                 hb.slot(x.t))
            ha.advance(x.t)
            out = self._conv_causal(f"{name}.c1", _Act(hb.slot(x.t), x.t, x.h, x.w, co), None, tmax, residual=h)
            return _Act(out, x.t, x.h, x.w, co)
        y = self._conv_causal(f"{name}.c0", x, self._rms(x.data, pk[f"{name}.g0"], ci, True), tmax)
        ya = _Act(y, x.t, x.h, x.w, co)
        out = self._conv_causal(f"{name}.c1", ya, self._rms(y, pk[f"{name}.g1"], co, True), tmax, residual=h)
        return _Act(out, x.t, x.h, x.w, co)

    def _attn(self, name, c, x):
        pk = self._packed[name]
        cp, dev = x.cp, x.data.device
        HW = x.h * x.w
        HWp = (HW + 63) // 64 * 64
        xn = torch.empty_like(x.data)
        kernels.vae_rms_silu(x.data, x.data.shape[0], cp, c, pk["g"], False, xn)
        out = torch.empty_like(x.data)
        comp = torch.zeros(HWp, cp, dtype=BF16, device=dev)
        S = torch.empty(HW, HWp, dtype=torch.float32, device=dev)
        Pm = torch.empty(HW, HWp, dtype=BF16, device=dev)
        vt = torch.empty(cp, HWp, dtype=BF16, device=dev)
        fr = x.P * cp
        for f in range(x.t):
            kernels.vae_gather(xn[f * x.P:(f + 1) * x.P], 1, x.h, x.w, cp, comp)
            qkv = kernels.gemm_bf16(comp, pk["wqkv"], pk["bqkv"])                   # [HWp, 3cp]
            kernels.gemm_f32(qkv, 3 * cp, qkv[:, cp:], 3 * cp, S, HWp, HW, HWp, cp)
            kernels.softmax_rows(S, HW, HW, HWp, 1.0 / math.sqrt(c), Pm)
            kernels.transpose_bf16(qkv[:, 2 * cp:], 3 * cp, HWp, cp, vt, HWp)
            o = kernels.gemm_bf16(Pm, vt)                                            # [HW, cp]
            y = kernels.gemm_bf16(o, pk["wo"], pk["bo"])
            kernels.vae_scatter_add(y, x.data.view(-1)[f * fr:(f + 1) * fr], 1, x.h, x.w, cp,
                                    out.view(-1)[f * fr:(f + 1) * fr])
        return _Act(out, x.t, x.h, x.w, c)

    def _resample(self, kind, name, c, x, tmax_in):
        dev = x.data.device
        if kind == "up3d":
            if name not in self._rep:
                self._rep.add(name)                                                  # first pass: no time conv
            else:
                src = x.data
                y = self._conv_causal(f"{name}.tc", x, lambda dest: dest.copy_(src), tmax_in)   # [t P, 2 cp]
                inter = torch.empty(2 * x.t * x.P, x.cp, dtype=BF16, device=dev)
                kernels.vae_time_interleave(y, x.t, x.P, x.cp, inter)
                x = _Act(inter, 2 * x.t, x.h, x.w, c)
        h2, w2 = 2 * x.h, 2 * x.w
        up = torch.empty(x.t * (h2 + 2) * (w2 + 2), x.cp, dtype=BF16, device=dev)
        kernels.vae_upsample2x(x.data, x.t, x.h, x.w, x.cp, up)
        out = self._conv_plain(f"{name}.rs", up, x.t, h2, w2)
        return _Act(out, x.t, h2, w2, c // 2)

    def _frame(self, xin):
        """One Decoder3d pass (vae2_1.py:428-477) on one latent frame (padded rows of conv2's output)."""
        pk = self._packed
        x = xin
        tmax = 1
        for kind, name, ci, co in self.layout:
            if kind == "conv":
                src = x.data
                out = self._conv_causal(name, x, lambda dest: dest.copy_(src), tmax)
                x = _Act(out, x.t, x.h, x.w, co)
            elif kind == "res":
                x = self._res(name, ci, co, x, tmax)
            elif kind == "attn":
                x = self._attn(name, ci, x)
            elif kind in ("up3d", "up2d"):
                x = self._resample(kind, name, ci, x, tmax)
                if kind == "up3d":
                    tmax *= 2
            else:
                out = self._conv_causal(f"{name}.c", x, self._rms(x.data, pk[f"{name}.g"], ci, True), tmax)
                x = _Act(out, x.t, x.h, x.w, 3)
        return x

    @torch.no_grad()
    def decode_latent(self, z, scale=None):
        """z [z_dim, T, h, w] -> frames [3, T', 8h, 8w] fp32 (not clamped), continuing this decoder's cache."""
        if self._packed is None:
            self.prepare()
        dev = self._packed["conv2"][0].device
        if scale is None:
            scale = [torch.tensor(LATENT_MEAN, dtype=BF16), 1.0 / torch.tensor(LATENT_STD, dtype=BF16)]
        zc = z.to(dev).float() / scale[1].to(dev).view(-1, 1, 1, 1) + scale[0].to(dev).view(-1, 1, 1, 1)
        c, T, h, w = zc.shape
        P = (h + 2) * (w + 2)
        zp = torch.zeros(T, h + 2, w + 2, _pad32(c), dtype=BF16, device=dev)      # padded rows of the latent
        zp[:, 1:-1, 1:-1, :c] = zc.permute(1, 2, 3, 0).to(BF16)
        x2 = self._conv_plain("conv2", zp.view(T * P, -1), T, h, w)
        outs = []
        for i in range(T):
            y = self._frame(_Act(x2[i * P:(i + 1) * P], 1, h, w, c))
            v = y.data.view(y.t, y.h + 2, y.w + 2, -1)[:, 1:-1, 1:-1, :3]
            outs.append(v.permute(3, 0, 1, 2).float())
        return torch.cat(outs, dim=1)

    def decode(self, z, scale=None):
        """WanVAE_.decode (:548-572): a fresh cache, then every latent frame."""
        self.clear_cache()
        out = self.decode_latent(z, scale)
        self.clear_cache()
        return out

    def decode_chunk(self, z, scale=None, first=False):
        """WanVAE_.decode_chunk (:574-596): consecutive chunks give the frames of one decode of the whole latent."""
        if first:
            self.clear_cache()
        return self.decode_latent(z, scale)


class Wan2_1_VAE:
    """Decode side of the reference's Wan2_1_VAE (vae2_1.py:647-700): the latent scale in bf16, outputs clamped to
    [-1, 1] in fp32. `vae_pth`: the reference's checkpoint (its encoder entries are ignored)."""

    def __init__(self, z_dim=16, vae_pth=None, dtype=BF16, device="cuda", dim=96, state_dict=None):
        self.dtype, self.device = dtype, device
        self.mean = torch.tensor(LATENT_MEAN, dtype=dtype, device=device)
        self.std = torch.tensor(LATENT_STD, dtype=dtype, device=device)
        self.scale = [self.mean, 1.0 / self.std]
        self.model = WanVAEDecoder(dim=dim, z_dim=z_dim)
        if state_dict is None and vae_pth is not None:
            state_dict = torch.load(vae_pth, map_location="cpu")
        if state_dict is not None:
            own = dict(self.model.named_parameters())
            missing = [k for k in own if k not in state_dict]
            if missing:
                raise ValueError(f"VAE checkpoint lacks {len(missing)} decoder tensors, e.g. {missing[:3]}")
            with torch.no_grad():
                for k, p in own.items():
                    p.copy_(state_dict[k].float())
        self.model.to(device)
        self.model.prepare()

    def decode(self, zs):
        return [self.model.decode(u, self.scale).clamp_(-1, 1) for u in zs]

    def decode_chunk(self, z, first):
        return self.model.decode_chunk(z, self.scale, first).clamp_(-1, 1)
