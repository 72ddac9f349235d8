"""MXFP8 block-scaled tcgen05 GEMMs (lbw_mx_*, lbw_layernorm_mod_mx, lbw_layernorm_affine_mx) against the
OCP-MX emulation of the oracle, through the C ABI."""
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
    assert rel_l2(out, ob.mx_matmul(a, w, b)) < 4e-3


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_mx_linear_gelu_emits_mx_codes(cuda_dev, fmt):
    import lbw_b200.kernels as K
    m, n, k = 333, 768, 512
    a, w, b = _ab(m, n, k, 5)
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d), fmt=fmt)
    wd, ws, _ = K.mx_quantize(w.to(d), fmt=fmt)
    oq, os_ = K.mx_buffers(m, n, d)
    K.mx_linear_gelu(ad, as_, wd, ws, b.to(d), oq, os_, fmt=fmt)
    u = ((omx.qdq(a, fmt) @ omx.qdq(w, fmt).t()).to(BF) + b).to(BF)
    g = F.gelu(u.float(), approximate="tanh").to(BF)
    q, s = omx.quantize(g, fmt)
    dt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    got = omx.dequantize(oq.cpu().view(dt), _untile(os_.cpu(), m, n))
    assert rel_l2(got, omx.dequantize(q, s)) < (1e-2 if fmt == "e4m3" else 2e-2)
    assert (_untile(os_.cpu(), m, n) == s).float().mean() > 0.99


def test_mx_linear_residual_e5m2(cuda_dev):
    import lbw_b200.kernels as K
    m, n, k = 260, 512, 768
    a, w, b = _ab(m, n, k, 9)
    d = cuda_dev
    x = torch.randn(m, n)
    gate = torch.randn(n) * 0.1
    ad, as_, _ = K.mx_quantize(a.to(d), fmt="e5m2")
    wd, ws, _ = K.mx_quantize(w.to(d), fmt="e5m2")
    xd = x.to(d)
    K.mx_linear_residual(ad, as_, wd, ws, b.to(d), xd, gate=gate.to(d), fmt="e5m2")
    y = ob.mx_matmul(a, w, b, "e5m2")
    assert rel_l2(xd.cpu() - x, y.float() * gate) < 5e-3


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


@pytest.mark.parametrize("c,fmt", [(128, "e4m3"), (1536, "e4m3"), (5120, "e4m3"), (1536, "e5m2")])
def test_layernorm_mod_mx(cuda_dev, c, fmt):
    import lbw_b200.kernels as K
    g = torch.Generator().manual_seed(11)
    m = 257
    x = torch.randn(m, c, generator=g) * 2 + 0.5
    s, t = torch.randn(c, generator=g) * 0.1, torch.randn(c, generator=g) * 0.1
    dq, ds = K.mx_buffers(m, c, cuda_dev)
    K.layernorm_mod_mx(x.to(cuda_dev), 1e-6, s.to(cuda_dev), t.to(cuda_dev), dq, ds, fmt=fmt)
    h = (ob.layer_norm(x, 1e-6) * (1 + s) + t).to(BF)
    q, se = omx.quantize(h, fmt)
    dt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    got = omx.dequantize(dq.cpu().view(dt), _untile(ds.cpu(), m, c))
    assert rel_l2(got, omx.dequantize(q, se)) < (2e-3 if fmt == "e4m3" else 4e-3)
    assert (_untile(ds.cpu(), m, c) == se).float().mean() > 0.99


@pytest.mark.parametrize("fmt", [None, "e5m2", "e2m1"])
def test_ffn_mx_mm_interface(cuda_dev, fmt):
    """ffn_mx.prequantize_weight / mm (the reference's operator names); fmt None = LINGBOT_MX_FP8's default E4M3."""
    import lbw_b200.ffn_mx as FM
    m, n, k = 200, 384, 512
    a, w, _ = _ab(m, n, k, 13)
    data, scales = FM.prequantize_weight(w.to(cuda_dev), fmt=fmt)
    out = FM.mm(a.to(cuda_dev), data, scales, fmt=fmt)
    assert rel_l2(out, omx.mx_linear(a, w, fmt or "e4m3")) < 4e-3


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


# ---- the other block Linears in MXFP8 (LINGBOT_LIN_MX): y = bf16(mm(x, W)) + b in bf16 ----------------------

def _mxq(t, d):
    import lbw_b200.kernels as K
    q, s, _ = K.mx_quantize(t.to(d))
    return q, s


def test_mx_qkv_proj_vs_emulation(cuda_dev):
    import lbw_b200.kernels as K
    m, c = 300, 512
    h, w, b = _ab(m, 3 * c, c, 31)
    d = cuda_dev
    q_raw = torch.empty(m, c, dtype=BF, device=d)
    k_raw = torch.empty(m, c, dtype=BF, device=d)
    ss = torch.full((2, m), 7.0, device=d)           # cleared by the call
    vbuf = torch.zeros(m + 40, c, dtype=BF, device=d)
    K.mx_qkv_proj(*_mxq(h, d), *_mxq(w, d), b.to(d), q_raw, k_raw, ss[0], ss[1], vbuf, v_row_off=17)
    ref = ob.mx_matmul(h, w, b)
    assert rel_l2(q_raw, ref[:, :c]) < 4e-3 and rel_l2(k_raw, ref[:, c:2 * c]) < 4e-3
    assert rel_l2(vbuf[17:17 + m], ref[:, 2 * c:]) < 4e-3
    assert not vbuf[:17].any() and not vbuf[17 + m:].any()
    for t, s in ((q_raw, ss[0]), (k_raw, ss[1])):
        assert rel_l2(s, t.float().pow(2).sum(1)) < 1e-5


def test_mx_linear_rowss_vs_emulation(cuda_dev):
    import lbw_b200.kernels as K
    m, n, k = 333, 768, 512
    a, w, b = _ab(m, n, k, 33)
    d = cuda_dev
    out = torch.empty(m, n, dtype=BF, device=d)
    ss = torch.full((m,), 3.0, device=d)
    K.mx_linear_rowss(*_mxq(a, d), *_mxq(w, d), b.to(d), out, ss)
    assert rel_l2(out, ob.mx_matmul(a, w, b)) < 4e-3
    assert rel_l2(ss, out.float().pow(2).sum(1)) < 1e-5


@pytest.mark.parametrize("m,n,k", [(260, 512, 1024), (1350, 1024, 512)])
def test_mx_linear_residual_film(cuda_dev, m, n, k):
    import lbw_b200.kernels as K
    a, w, b = _ab(m, n, k, 35)
    g = torch.Generator().manual_seed(36)
    x = torch.randn(m, n, generator=g)
    gate = torch.randn(n, generator=g) * 0.1
    fs = (torch.randn(m, n, generator=g) * 0.1).to(BF)
    ft = (torch.randn(m, n, generator=g) * 0.1).to(BF)
    d = cuda_dev
    xd = x.to(d)
    K.mx_linear_residual(*_mxq(a, d), *_mxq(w, d), b.to(d), xd, gate=gate.to(d), film_scale=fs.to(d),
                         film_shift=ft.to(d))
    x1 = x + ob.mx_matmul(a, w, b).float() * gate
    ref = (1.0 + fs) * x1 + ft
    assert rel_l2(xd, ref) < 1e-4 and rel_l2(xd.cpu() - x, ref - x) < 5e-3


def test_mx_linear_act(cuda_dev):
    import lbw_b200.kernels as K
    m, n, k = 200, 512, 512
    a, w, b = _ab(m, n, k, 37)
    c = (torch.randn(m, n, generator=torch.Generator().manual_seed(38))).to(BF)
    d = cuda_dev
    aq, w_mx = _mxq(a, d), _mxq(w, d)
    y = ob.mx_matmul(a, w, b)
    h = K.mx_linear_act(*aq, *w_mx, b.to(d), silu=True)
    assert rel_l2(h, F.silu(y.float()).to(BF)) < 5e-3
    h2 = K.mx_linear_act(*aq, *w_mx, b.to(d), addend=c.to(d))
    assert rel_l2(h2, (y + c).to(BF)) < 5e-3


@pytest.mark.parametrize("c", [512, 5120])
def test_layernorm_affine_mx(cuda_dev, c):
    import lbw_b200.kernels as K
    g = torch.Generator().manual_seed(39)
    m = 131
    x = torch.randn(m, c, generator=g) * 2 - 0.3
    w3, b3 = 1 + torch.randn(c, generator=g) * 0.1, torch.randn(c, generator=g) * 0.1
    dq, ds = K.mx_buffers(m, c, cuda_dev)
    K.layernorm_affine_mx(x.to(cuda_dev), 1e-6, w3.to(cuda_dev), b3.to(cuda_dev), dq, ds)
    h = ob.layer_norm(x, 1e-6, w3, b3).to(BF)
    q, se = omx.quantize(h)
    got = omx.dequantize(dq.cpu().view(torch.float8_e4m3fn), _untile(ds.cpu(), m, c))
    assert rel_l2(got, omx.dequantize(q, se)) < 2e-3


# ---- the other element formats: E5M2 (LINGBOT_MX_FP8=float8_e5m2, kernels/ffn_mx.py:8, :18) and E2M1 (MXFP4) ----

def _codes(q, fmt):
    """Oracle element values -> the bytes the GPU stores (E2M1: packed nibbles, element 2i low)."""
    if fmt == "e2m1":
        return omx.e2m1_pack(omx.e2m1_codes(q))
    return q.view(torch.uint8)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m1"])
def test_mx_quantize_formats_bit_exact(cuda_dev, fmt):
    """Codes, E8M0 scales (tiled) and dequantised values bit-exact with the OCP MX emulation, over 6 decades of
    magnitude, an all-zero block and a block that saturates the element format."""
    import lbw_b200.kernels as K
    g = torch.Generator().manual_seed(41)
    rows, k = 300, 512
    x = (torch.randn(rows, k, generator=g) * torch.logspace(-3, 3, rows).view(-1, 1)).to(BF)
    x[5] = 0
    x[7, :32] = 1000.0
    x[9, 64:96] = torch.linspace(-7.0, 7.0, 32)     # E2M1 ties and the +-6 saturation
    data, scales, deq = K.mx_quantize(x.to(cuda_dev), dequant=True, fmt=fmt)
    q, s = omx.quantize(x, fmt)
    assert torch.equal(data.cpu(), _codes(q, fmt))
    assert torch.equal(scales.cpu(), omx.scales_tiled(s, k))
    assert torch.equal(deq.cpu().float(), omx.dequantize(q, s))


@pytest.mark.parametrize("fmt", ["e5m2", "e2m1"])
@pytest.mark.parametrize("m,n,k", [(128, 256, 256), (300, 512, 768), (77, 384, 512), (1350, 1024, 1024),
                                   (1000, 1536, 1536)])
def test_mx_linear_formats_vs_emulation(cuda_dev, fmt, m, n, k):
    """The block-scaled GEMM in E5M2 (kind::mxf8f6f4) and E2M1 (kind::mxf4) against the emulation: the same
    quantised operands, so only the fp32 summation order differs before the bf16 rounding."""
    import lbw_b200.kernels as K
    a, w, b = _ab(m, n, k, 7 * m + n + k)
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d), fmt=fmt)
    wd, ws, _ = K.mx_quantize(w.to(d), fmt=fmt)
    out = K.mx_linear(ad, as_, wd, ws, b.to(d), fmt=fmt)
    ref = (omx.mx_linear(a, w, fmt).float() + b.float()).to(BF)
    assert rel_l2(out, ref) < 4e-3


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m1"])
def test_mx_wide_tiles_with_a_half_scale_block(cuda_dev, monkeypatch, fmt):
    """256-wide tiles (forced with LBW_GEMM_TILE_N) where N = 640 is an odd number of 128-row weight blocks: the
    last tile's second scale block does not exist (the kernel reuses the first one for those rows) and its columns
    past N are dropped by every epilogue. The automatic choice runs 128-wide tiles at these shapes, so only the
    override reaches this path."""
    import lbw_b200.kernels as K
    monkeypatch.setenv("LBW_GEMM_TILE_N", "256")
    m, n, k = 300, 640, 768
    a, w, b = _ab(m, n, k, 31)
    d = cuda_dev
    ad, as_, _ = K.mx_quantize(a.to(d), fmt=fmt)
    wd, ws, _ = K.mx_quantize(w.to(d), fmt=fmt)
    out = K.mx_linear(ad, as_, wd, ws, b.to(d), fmt=fmt)
    y = omx.mx_linear(a, w, fmt)
    assert rel_l2(out, (y.float() + b.float()).to(BF)) < 4e-3
    if fmt == "e2m1":
        return
    g = torch.Generator().manual_seed(32)
    x = torch.randn(m, n, generator=g)
    gate = torch.randn(n, generator=g) * 0.1
    xd = x.to(d)
    K.mx_linear_residual(ad, as_, wd, ws, b.to(d), xd, gate=gate.to(d), fmt=fmt)
    assert rel_l2(xd.cpu() - x, ob.mx_matmul(a, w, b, fmt).float() * gate) < 5e-3
    oq, os_ = K.mx_buffers(m, n, d, fmt=fmt)
    K.mx_linear_gelu(ad, as_, wd, ws, b.to(d), oq, os_, fmt=fmt)
    u = (y.to(BF) + b).to(BF)
    q, s = omx.quantize(F.gelu(u.float(), approximate="tanh").to(BF), fmt)
    dt = torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2
    got = omx.dequantize(oq.cpu().view(dt), _untile(os_.cpu(), m, n))
    assert rel_l2(got, omx.dequantize(q, s)) < (1e-2 if fmt == "e4m3" else 2e-2)


def test_mx_formats_reject_bad_shapes(cuda_dev):
    import lbw_b200.kernels as K
    d = cuda_dev
    a = torch.zeros(128, 384, dtype=BF, device=d)
    ad, as_, _ = K.mx_quantize(a, fmt="e2m1")      # 384 % 128 == 0: fine for the quantiser
    with pytest.raises(ValueError, match="multiple of 256"):
        K.mx_linear(ad, as_, ad, as_, fmt="e2m1")      # ... but an E2M1 GEMM needs k % 256 == 0
    with pytest.raises(ValueError, match="element format"):
        K.mx_quantize(a, fmt="e3m2")
