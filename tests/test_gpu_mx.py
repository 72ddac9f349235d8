"""MXFP8 block-scaled tcgen05 GEMMs (lbw_mx_linear*, lbw_layernorm_mod_mx) against the OCP-MX emulation
of the oracle, through the C ABI."""
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_l2
from oracle import block as ob
from oracle import mx as omx

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _ab(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(BF)
    w = (torch.randn(n, k, generator=g) * 0.05).to(BF)
    b = (torch.randn(n, generator=g) * 0.05).to(BF)
    return a, w, b


@pytest.mark.parametrize("m,n,k", [(128, 256, 128), (300, 512, 640), (77, 384, 256), (4680, 1536, 1536),
                                   (1000, 13824 // 4, 5120 // 4),
                                   (1350, 5120, 1024),    # 1,350 rows (8-way split of 720p): 128-wide tiles,
                                   (1350, 5120, 1152),    # ... an odd number of K blocks: 256-wide tiles
                                   (1350, 2560, 2048)])   # ... two K blocks per stage over 8 stages
def test_mx_linear_vs_emulation(cuda_dev, m, n, k):
    import lbw_b200.kernels as K
    a, w, b = _ab(m, n, k, m + n + k)
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d))
    wd, ws, _ = K.mx_quantize(w.to(d))
    out = K.mx_linear(ad, as_, wd, ws, b.to(d))
    ref = (omx.qdq(a) @ omx.qdq(w).t() + b.float()).to(BF)
    assert rel_l2(out, ref) < 4e-3


def test_mx_linear_gelu_emits_mx_codes(cuda_dev):
    import lbw_b200.kernels as K
    m, n, k = 333, 768, 512
    a, w, b = _ab(m, n, k, 5)
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d))
    wd, ws, _ = K.mx_quantize(w.to(d))
    oq, os_ = K.mx_buffers(m, n, d)
    K.mx_linear_gelu(ad, as_, wd, ws, b.to(d), oq, os_)
    u = ((omx.qdq(a) @ omx.qdq(w).t()).to(BF) + b).to(BF)
    g = F.gelu(u.float(), approximate="tanh").to(BF)
    q, s = omx.quantize(g)
    got = omx.dequantize(oq.cpu().view(torch.float8_e4m3fn), _untile(os_.cpu(), m, n))
    assert rel_l2(got, omx.dequantize(q, s)) < 1e-2
    assert (_untile(os_.cpu(), m, n) == s).float().mean() > 0.99


def _untile(tiled, rows, k):
    r = torch.arange(rows).view(-1, 1).expand(rows, k // 32)
    j = torch.arange(k // 32).view(1, -1).expand(rows, k // 32)
    return tiled[omx.sf_offset(r, j, k)].to(torch.int32) - 127


def test_mx_linear_residual(cuda_dev):
    import lbw_b200.kernels as K
    m, n, k = 260, 512, 1024
    a, w, b = _ab(m, n, k, 7)
    g = torch.Generator().manual_seed(8)
    x = torch.randn(m, n, generator=g)
    gate = torch.randn(n, generator=g) * 0.1
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d))
    wd, ws, _ = K.mx_quantize(w.to(d))
    xd = x.to(d)
    K.mx_linear_residual(ad, as_, wd, ws, b.to(d), xd, gate=gate.to(d))
    y = (omx.qdq(a) @ omx.qdq(w).t() + b.float()).to(BF)
    ref = x + y.float() * gate
    assert rel_l2(xd - x.to(d), ref - x) < 5e-3


@pytest.mark.parametrize("c", [128, 1536, 5120])
def test_layernorm_mod_mx(cuda_dev, c):
    import lbw_b200.kernels as K
    g = torch.Generator().manual_seed(11)
    m = 257
    x = torch.randn(m, c, generator=g) * 2 + 0.5
    s, t = torch.randn(c, generator=g) * 0.1, torch.randn(c, generator=g) * 0.1
    dq, ds = K.mx_buffers(m, c, cuda_dev)
    K.layernorm_mod_mx(x.to(cuda_dev), 1e-6, s.to(cuda_dev), t.to(cuda_dev), dq, ds)
    h = (ob.layer_norm(x, 1e-6) * (1 + s) + t).to(BF)
    q, se = omx.quantize(h)
    got = omx.dequantize(dq.cpu().view(torch.float8_e4m3fn), _untile(ds.cpu(), m, c))
    assert rel_l2(got, omx.dequantize(q, se)) < 2e-3


def test_ffn_mx_mm_interface(cuda_dev):
    import lbw_b200.ffn_mx as FM
    m, n, k = 200, 384, 512
    a, w, _ = _ab(m, n, k, 13)
    data, scales = FM.prequantize_weight(w.to(cuda_dev))
    out = FM.mm(a.to(cuda_dev), data, scales)
    assert rel_l2(out, omx.mx_linear(a, w)) < 4e-3


def test_mx_linear_residual_narrow_tiles(cuda_dev):
    import lbw_b200.kernels as K
    m, n, k = 1350, 5120, 512
    a, w, b = _ab(m, n, k, 17)
    x = torch.randn(m, n, generator=torch.Generator().manual_seed(18))
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d))
    wd, ws, _ = K.mx_quantize(w.to(d))
    xd = x.to(d)
    K.mx_linear_residual(ad, as_, wd, ws, b.to(d), xd)
    y = (omx.qdq(a) @ omx.qdq(w).t() + b.float()).to(BF)
    assert rel_l2(xd - x.to(d), y.float()) < 5e-3
