"""The Wan 2.1 VAE decoder on a B200: its kernels against fp32 torch, and the whole decode against the reference's
own WanVAE_.decode / decode_chunk (tests/golden/vae_decode.pt), through the C ABI."""
import math

import pytest
import torch
import torch.nn.functional as F

from conftest import load_golden, max_abs, rel_l2
from oracle import vae as ov

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _g(seed):
    return torch.Generator().manual_seed(seed)


def _padded(x, cp):
    """x [T, C, h, w] fp32 -> padded channels-last rows [T * (h + 2) * (w + 2), cp] bf16."""
    T, C, h, w = x.shape
    out = torch.zeros(T, h + 2, w + 2, cp, dtype=BF)
    out[:, 1:-1, 1:-1, :C] = x.permute(0, 2, 3, 1).to(BF)
    return out.reshape(T * (h + 2) * (w + 2), cp)


def _unpad(rows, T, h, w, C):
    return rows.reshape(T, h + 2, w + 2, -1)[:, 1:-1, 1:-1, :C].permute(0, 3, 1, 2).float()


def _pack(wt, cip, cop):
    co, ci = wt.shape[:2]
    wp = torch.zeros(cop, cip, *wt.shape[2:])
    wp[:co, :ci] = wt
    return wp.permute(0, 2, 3, 4, 1).reshape(cop, -1).to(BF).contiguous()


@pytest.mark.parametrize("k,t,ci,co,h,w", [((3, 3, 3), 2, 40, 70, 5, 7), ((3, 3, 3), 1, 64, 128, 9, 4),
                                           ((1, 3, 3), 3, 100, 50, 6, 6), ((1, 1, 1), 2, 64, 64, 3, 5),
                                           ((3, 1, 1), 2, 64, 256, 4, 4),
                                           ((3, 3, 3), 2, 64, 192, 5, 6),    # 192-wide tiles
                                           ((1, 1, 1), 1, 128, 384, 4, 4),   # two 192-wide tiles
                                           ((3, 3, 3), 2, 96, 3, 4, 6),      # the head: 64-wide tiles
                                           ((3, 3, 3), 2, 16, 32, 3, 4),     # 16 stored channels in a 64 block
                                           ((3, 3, 3), 2, 96, 96, 6, 9),     # the full-resolution level (dim 96)
                                           ((3, 3, 3), 1, 192, 96, 4, 5),    # upsampled 192 -> 96 channels
                                           ((3, 3, 3), 1, 384, 384, 3, 4),   # the lowest levels (dim 96)
                                           ((3, 3, 3), 2, 32, 32, 3, 4),     # 32 channels (dim 32)
                                           ((3, 3, 3), 1, 96, 192, 4, 5),    # 96 -> 192 channels, 192-wide tiles
                                           ((1, 1, 1), 2, 32, 256, 9, 9)])   # 32 stored channels in a 64 block
def test_vae_conv_vs_torch(cuda_dev, k, t, ci, co, h, w):
    import lbw_b200.kernels as K
    g = _g(ci + co + t)
    kt, kh, kw = k
    tin = t + kt - 1
    x = torch.randn(tin, ci, h, w, generator=g).to(BF).float()
    wt = (torch.randn(co, ci, kt, kh, kw, generator=g) / math.sqrt(ci * kt * kh * kw)).to(BF).float()
    b = (torch.randn(co, generator=g) * 0.1).to(BF)
    # stored channels: a multiple of 8; K blocks of 64 read past them as zeros (TMA out-of-bounds fill)
    cis, cop = (ci + 7) // 8 * 8, (co + 31) // 32 * 32
    cik = (cis + 63) // 64 * 64
    P = (h + 2) * (w + 2)
    d = cuda_dev
    xr = _padded(x, cis).to(d)
    res = torch.randn(t * P, cop, generator=g).to(BF)
    bp = torch.zeros(cop, dtype=BF)
    bp[:co] = b
    out = torch.full((t * P, cop), 7.0, dtype=BF, device=d)
    K.vae_conv(xr, tin * P, cis, _pack(wt, cik, cop).to(d), bp.to(d), cop, k, t, h, w, out, residual=res.to(d))
    ref = F.conv3d(x.permute(1, 0, 2, 3).unsqueeze(0), wt, b.float(), padding=(0, kh // 2, kw // 2))[0]
    ref = ref.permute(1, 0, 2, 3)                                            # [t, co, h, w]
    got = _unpad(out.cpu(), t, h, w, co)
    resid = _unpad(res, t, h, w, co)
    assert rel_l2(got - resid, ref) < 1e-2
    rows = out.cpu().reshape(t, h + 2, w + 2, cop)
    assert not rows[:, 0].any() and not rows[:, -1].any() and not rows[:, :, 0].any() and not rows[:, :, -1].any()


@pytest.mark.parametrize("ci,co,t", [(96, 96, 2), (64, 192, 1), (16, 32, 2)])
def test_vae_conv_rms_fused(cuda_dev, ci, co, t):
    """The first ResidualBlock convolution with its RMS_norm + SiLU in the epilogue equals the convolution followed
    by the separate RMS + SiLU kernel (128-, 192- and 256-wide tiles holding whole rows)."""
    import lbw_b200.kernels as K
    g = _g(ci + co)
    h, w = 5, 6
    x = torch.randn(t + 2, ci, h, w, generator=g).to(BF).float()
    wt = (torch.randn(co, ci, 3, 3, 3, generator=g) / math.sqrt(ci * 27)).to(BF).float()
    b = (torch.randn(co, generator=g) * 0.1).to(BF)
    gamma = 1 + 0.1 * torch.randn(co, generator=g)
    cis, cop = (ci + 7) // 8 * 8, (co + 31) // 32 * 32
    cik = (cis + 63) // 64 * 64
    P = (h + 2) * (w + 2)
    d = cuda_dev
    xr = _padded(x, cis).to(d)
    wk = _pack(wt, cik, cop).to(d)
    bp = torch.zeros(cop, dtype=BF)
    bp[:co] = b
    gp = torch.zeros(cop)
    gp[:co] = gamma
    fused = torch.full((t * P, cop), 3.0, dtype=BF, device=d)
    K.vae_conv_rms(xr, (t + 2) * P, cis, wk, bp.to(d), cop, (3, 3, 3), t, h, w, gp.to(d), co, fused)
    y = torch.empty(t * P, cop, dtype=BF, device=d)
    K.vae_conv(xr, (t + 2) * P, cis, wk, bp.to(d), cop, (3, 3, 3), t, h, w, y)
    sep = torch.empty_like(y)
    K.vae_rms_silu(y, t * P, cop, co, gp.to(d), True, sep)
    assert rel_l2(fused.float(), sep.float()) < 1e-2
    ref = F.conv3d(x.permute(1, 0, 2, 3).unsqueeze(0), wt, b.float(), padding=(0, 1, 1))[0].permute(1, 0, 2, 3)
    ref = F.silu(ov.rms_norm(ref.to(BF).float(), gamma))
    assert rel_l2(_unpad(fused.cpu(), t, h, w, co), ref) < 2e-2
    assert not fused.cpu().reshape(t, h + 2, w + 2, cop)[:, 0].any()


def test_vae_rms_silu(cuda_dev):
    import lbw_b200.kernels as K
    g = _g(3)
    x = torch.randn(2, 96, 4, 5, generator=g) * 3
    gamma = 1 + 0.1 * torch.randn(96, generator=g)
    cp = 128
    xr = _padded(x, cp)
    gp = torch.zeros(cp)
    gp[:96] = gamma
    for silu in (True, False):
        out = torch.empty_like(xr, device=cuda_dev)
        K.vae_rms_silu(xr.to(cuda_dev), xr.shape[0], cp, 96, gp.to(cuda_dev), silu, out)
        xb = _unpad(xr, 2, 4, 5, 96)
        ref = ov.rms_norm(xb, gamma)
        ref = F.silu(ref) if silu else ref
        assert rel_l2(_unpad(out.cpu(), 2, 4, 5, 96), ref) < 1e-2
        assert not out.cpu().reshape(2, 6, 7, cp)[:, 0].any()


def test_vae_upsample_interleave_gather_scatter(cuda_dev):
    import lbw_b200.kernels as K
    g = _g(4)
    d = cuda_dev
    x = torch.randn(2, 64, 3, 5, generator=g)
    xr = _padded(x, 64).to(d)
    up = torch.empty(2 * 8 * 12, 64, dtype=BF, device=d)
    K.vae_upsample2x(xr, 2, 3, 5, 64, up)
    ref = F.interpolate(x.to(BF).float(), scale_factor=(2.0, 2.0), mode="nearest-exact")
    assert torch.equal(_unpad(up.cpu(), 2, 6, 10, 64), ref)
    assert not up.cpu().reshape(2, 8, 12, 64)[:, :, 0].any()
    y = torch.randn(2 * 5 * 7, 128, generator=g).to(BF).to(d)             # 2 frames of P = 35 rows, [c | c]
    inter = torch.empty(4 * 35, 64, dtype=BF, device=d)
    K.vae_time_interleave(y, 2, 35, 64, inter)
    yv = y.cpu().reshape(2, 35, 2, 64)
    assert torch.equal(inter.cpu().reshape(2, 2, 35, 64), yv.permute(0, 2, 1, 3))
    comp = torch.empty(2 * 15, 64, dtype=BF, device=d)
    K.vae_gather(xr, 2, 3, 5, 64, comp)
    assert torch.equal(comp.cpu().float(), x.to(BF).float().permute(0, 2, 3, 1).reshape(30, 64))
    out = torch.empty_like(xr)
    K.vae_scatter_add(comp, xr, 2, 3, 5, 64, out)
    assert torch.equal(_unpad(out.cpu(), 2, 3, 5, 64), (x.to(BF) + x.to(BF)).float())


def test_attention_pieces(cuda_dev):
    """fp32-output GEMM, row softmax with padded columns, and the bf16 transpose of the mid-block attention."""
    import lbw_b200.kernels as K
    g = _g(5)
    d = cuda_dev
    n, npad, c = 200, 256, 128
    q = torch.randn(npad, 3 * c, generator=g).to(BF)
    S = torch.empty(n, npad, device=d)
    qd = q.to(d)
    K.gemm_f32(qd, 3 * c, qd[:, c:], 3 * c, S, npad, n, npad, c)
    ref = q[:n, :c].float() @ q[:, c:2 * c].float().t()
    assert rel_l2(S.cpu(), ref) < 1e-5
    Pm = torch.empty(n, npad, dtype=BF, device=d)
    K.softmax_rows(S, n, n, npad, 0.1, Pm)
    pref = torch.softmax(ref[:, :n] * 0.1, dim=-1)
    assert rel_l2(Pm.cpu()[:, :n].float(), pref) < 1e-2 and not Pm.cpu()[:, n:].any()
    vt = torch.empty(c, npad, dtype=BF, device=d)
    K.transpose_bf16(qd[:, 2 * c:], 3 * c, npad, c, vt, npad)
    assert torch.equal(vt.cpu(), q[:, 2 * c:].t())


def _decoder(g, dev):
    import lbw_b200.vae as V
    p = ov.make_params(g["seed"], **g["cfg"])
    m = V.WanVAEDecoder(dim=g["cfg"]["dim"])
    sd = m.state_dict()
    for k, v in p.items():
        sd[k] = v
    m.load_state_dict(sd)
    m.to(dev).prepare()
    return m


def test_vae_decode_vs_reference_golden(cuda_dev):
    """Whole decode of a 3-frame latent (9 frames out) against the reference's fp32 WanVAE_.decode. The B200 path
    keeps activations in bf16 (fp32 accumulation): a bf16 run of the same math on CPU differs from the fp32
    reference by 1.7e-2 relative L2 (max 0.043), hence the tolerance."""
    g = load_golden("vae_decode")
    m = _decoder(g, cuda_dev)
    out = m.decode(g["z"], ov.latent_scale()).clamp(-1, 1).cpu()
    assert out.shape == g["out"].shape and torch.isfinite(out).all()
    assert rel_l2(out, g["out"]) < 3e-2 and max_abs(out, g["out"]) < 0.15


def test_vae_decode_chunk_streams_like_one_decode(cuda_dev):
    """decode_chunk over 2 + 1 latent frames continues every causal cache: the same frames as one decode."""
    g = load_golden("vae_decode")
    m = _decoder(g, cuda_dev)
    full = m.decode(g["z"], ov.latent_scale())
    a = m.decode_chunk(g["z"][:, :2], ov.latent_scale(), first=True)
    b = m.decode_chunk(g["z"][:, 2:], ov.latent_scale())
    assert torch.equal(torch.cat([a, b], dim=1), full)
    assert rel_l2(torch.cat([a, b], dim=1).clamp(-1, 1).cpu(), g["out_chunks"]) < 3e-2


def test_wan21_vae_wrapper_decode(cuda_dev):
    """Wan2_1_VAE (the reference's decode interface) from a full WanVAE_-style state dict: encoder entries are
    ignored, the bf16 latent scale is applied, frames come back clamped to [-1, 1]."""
    import lbw_b200.vae as V
    g = load_golden("vae_decode")
    sd = dict(ov.make_params(g["seed"], **g["cfg"]))
    sd["encoder.conv1.weight"] = torch.zeros(4, 3, 3, 3, 3)       # present in the reference checkpoint, unused here
    vae = V.Wan2_1_VAE(z_dim=16, dim=g["cfg"]["dim"], device=cuda_dev, state_dict=sd)
    out = vae.decode([g["z"]])[0].cpu()
    assert out.shape == g["out"].shape and float(out.abs().max()) <= 1.0
    assert rel_l2(out, g["out"]) < 3e-2
    a = vae.decode_chunk(g["z"][:, :2], True)
    b = vae.decode_chunk(g["z"][:, 2:], False)
    assert torch.equal(torch.cat([a, b], dim=1).cpu(), out)
