"""Kernel parity on a B200: every liblbw.so kernel against the CPU oracle (or an fp32 torch reference for
the plain GEMM) on seeded inputs, through the C ABI."""
import math

import pytest
import torch
import torch.nn.functional as F

from conftest import max_abs, rel_l2
from oracle import block as ob
from oracle import mx as omx

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _g(seed):
    return torch.Generator().manual_seed(seed)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (200, 512, 320), (1000, 768, 1536), (4680, 1536, 1536),
                                   (77, 96, 128), (1350, 5120, 512)])   # the last one runs 128-wide tiles
def test_gemm_bf16(cuda_dev, m, n, k):
    import lbw_b200.kernels as K
    g = _g(m + n + k)
    a = torch.randn(m, k, generator=g).to(BF)
    w = (torch.randn(n, k, generator=g) * 0.05).to(BF)
    b = (torch.randn(n, generator=g) * 0.1).to(BF)
    out = K.gemm_bf16(a.to(cuda_dev), w.to(cuda_dev), b.to(cuda_dev))
    ref = a.float() @ w.float().t() + b.float()
    assert rel_l2(out, ref) < 4e-3
    assert max_abs(out, ref) < 2e-2 * float(ref.abs().max())


def test_qkv_proj_regions_and_row_ss(cuda_dev):
    import lbw_b200.kernels as K
    g = _g(3)
    m, c = 300, 512
    h = torch.randn(m, c, generator=g).to(BF)
    w = (torch.randn(3 * c, c, generator=g) * 0.02).to(BF)
    b = (torch.randn(3 * c, generator=g) * 0.02).to(BF)
    d = cuda_dev
    q, k = torch.empty(m, c, dtype=BF, device=d), torch.empty(m, c, dtype=BF, device=d)
    ss = torch.empty(2, m, device=d)
    v_dst = torch.full((m + 64, c), float("nan"), dtype=BF, device=d)
    K.qkv_proj(h.to(d), w.to(d), b.to(d), q, k, ss[0], ss[1], v_dst, v_row_off=64)
    ref = ob.linear(h, w, b)
    assert rel_l2(q, ref[:, :c]) < 4e-3 and rel_l2(k, ref[:, c:2 * c]) < 4e-3
    assert rel_l2(v_dst[64:], ref[:, 2 * c:]) < 4e-3
    assert torch.isnan(v_dst[:64].float()).all()
    assert rel_l2(ss[0], q.float().pow(2).sum(1)) < 1e-5
    assert rel_l2(ss[1], k.float().pow(2).sum(1)) < 1e-5


def test_linear_residual_gate_and_film(cuda_dev):
    import lbw_b200.kernels as K
    g = _g(4)
    m, n, k = 260, 512, 256
    a = torch.randn(m, k, generator=g).to(BF)
    w = (torch.randn(n, k, generator=g) * 0.05).to(BF)
    b = (torch.randn(n, generator=g) * 0.05).to(BF)
    x = torch.randn(m, n, generator=g)
    gate = torch.randn(n, generator=g) * 0.1
    fs, ft = (torch.randn(m, n, generator=g) * 0.1).to(BF), (torch.randn(m, n, generator=g) * 0.1).to(BF)
    d = cuda_dev
    xd = x.to(d)
    K.linear_residual(a.to(d), w.to(d), b.to(d), xd, gate=gate.to(d), film_scale=fs.to(d), film_shift=ft.to(d))
    y = ob.linear(a, w, b)
    ref = (1.0 + fs) * (x + y.float() * gate) + ft
    assert rel_l2(xd, ref) < 1e-4 and rel_l2(xd - x.to(d), ref - x) < 5e-3
    xd2 = x.to(d)
    K.linear_residual(a.to(d), w.to(d), None, xd2)
    assert rel_l2(xd2 - x.to(d), ob.linear(a, w, None).float()) < 5e-3


@pytest.mark.parametrize("width", [128, 256])
@pytest.mark.parametrize("m,n,k", [(300, 640, 512), (77, 96, 128), (200, 160, 256)])
def test_bf16_gemm_epilogues_at_both_tile_widths(cuda_dev, monkeypatch, width, m, n, k):
    """Each tile width (forced with LBW_GEMM_TILE_N) at N not a multiple of 256, so that the last tile is cut inside
    its columns: the automatic choice picks one width per shape, and the shapes of the other tests are whole
    256-wide tiles wherever 256 is chosen. The store, residual + FiLM and row-sum-of-squares epilogues."""
    import lbw_b200.kernels as K
    monkeypatch.setenv("LBW_GEMM_TILE_N", str(width))
    g = _g(m + n + k + width)
    a = torch.randn(m, k, generator=g).to(BF)
    w = (torch.randn(n, k, generator=g) * 0.05).to(BF)
    b = (torch.randn(n, generator=g) * 0.05).to(BF)
    x = torch.randn(m, n, generator=g)
    gate = torch.randn(n, generator=g) * 0.1
    fs, ft = (torch.randn(m, n, generator=g) * 0.1).to(BF), (torch.randn(m, n, generator=g) * 0.1).to(BF)
    d = cuda_dev
    y = ob.linear(a, w, b)
    out = K.gemm_bf16(a.to(d), w.to(d), b.to(d))
    assert rel_l2(out, y) < 4e-3
    xd = x.to(d)
    K.linear_residual(a.to(d), w.to(d), b.to(d), xd, gate=gate.to(d), film_scale=fs.to(d), film_shift=ft.to(d))
    ref = (1.0 + fs) * (x + y.float() * gate) + ft
    assert rel_l2(xd, ref) < 1e-4
    out2 = torch.empty(m, n, dtype=BF, device=d)
    ss = torch.empty(m, device=d)
    K.linear_rowss(a.to(d), w.to(d), b.to(d), out2, ss)
    assert rel_l2(out2, y) < 4e-3
    assert rel_l2(ss, out2.float().pow(2).sum(1)) < 1e-5


@pytest.mark.parametrize("qdq", [False, True])
def test_linear_gelu(cuda_dev, qdq):
    import lbw_b200.kernels as K
    g = _g(5)
    m, n, k = 333, 768, 512
    a = torch.randn(m, k, generator=g).to(BF)
    w = (torch.randn(n, k, generator=g) * 0.05).to(BF)
    b = (torch.randn(n, generator=g) * 0.05).to(BF)
    out = torch.empty(m, n, dtype=BF, device=cuda_dev)
    K.linear_gelu(a.to(cuda_dev), w.to(cuda_dev), b.to(cuda_dev), out, qdq)
    # plain Linear: one rounding of acc + b; the MX-emulating variant rounds the matmul first (ffn_mx.mm + bias)
    u = ((a.float() @ w.float().t()).to(BF) + b).to(BF) if qdq else ob.linear(a, w, b)
    ref = F.gelu(u.float(), approximate="tanh").to(BF)
    if qdq:
        ref = omx.qdq(ref)
    assert rel_l2(out, ref) < 1e-2


def _attn_case(lq, rows, heads, seed, qscale=1.0):
    g = _g(seed)
    q = (torch.randn(lq, heads, 128, generator=g) * qscale).to(BF)
    ks = [torch.randn(r, heads, 128, generator=g).to(BF) for r in rows]
    vs = [torch.randn(r, heads, 128, generator=g).to(BF) for r in rows]
    return q, ks, vs


@pytest.mark.parametrize("lq,rows,heads,qscale", [
    (256, [256], 1, 1.0),
    (300, [200, 77, 128], 2, 1.0),          # ragged query tile and ragged KV tiles
    (129, [1000], 3, 3.0),                  # peaked: logits up to ~50 -> running-max rescales
    (512, [72, 72, 72, 72, 72, 72, 72], 2, 2.0),   # 7 chunks (the 21-frame window)
    (40, [4680, 4680, 4680], 1, 0.5),
])
def test_chunk_attention(cuda_dev, lq, rows, heads, qscale):
    import lbw_b200.kernels as K
    q, ks, vs = _attn_case(lq, rows, heads, lq + sum(rows), qscale)
    d = cuda_dev
    out = K.chunk_attention(q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs])
    ref = ob.attention(q, torch.cat(ks), torch.cat(vs))
    assert rel_l2(out.view(lq, heads, 128), ref) < 1e-2
    assert max_abs(out.view(lq, heads, 128), ref) < 5e-2


@pytest.mark.parametrize("lq,rows,heads,bias", [
    (70, [128, 77], 2, False),        # lone query tile: ping-pong over 2 key tiles, the odd one ragged
    (70, [100], 1, False),            # one key tile: slot 1 stays empty
    (128, [300, 300, 300], 2, True),  # full lone tile, 9 key tiles (odd count), key bias
    (1350, [256] * 7, 2, False),      # 8-rank c4 rows per head: five two-tile CTAs + a 70-row lone tile
])
def test_chunk_attention_lone_tile_ping_pong(cuda_dev, lq, rows, heads, bias):
    """A CTA whose second query tile is past the last row splits its key tiles between two softmax slots and
    merges the two partial softmaxes; direct output and split-KV partials both match fp32."""
    import lbw_b200.kernels as K
    q, ks, vs = _attn_case(lq, rows, heads, 41 + lq, qscale=2.0)
    kb = None
    if bias:
        kb = torch.zeros(sum(rows))
        kb[::3] = math.log(5.0)
    d = cuda_dev
    kd, vd = [k.to(d) for k in ks], [v.to(d) for v in vs]
    out = K.chunk_attention(q.to(d), kd, vd, key_bias=None if kb is None else kb.to(d))
    ref = ob.attention(q, torch.cat(ks), torch.cat(vs), key_bias=kb)
    assert rel_l2(out.view(lq, heads, 128), ref) < 1e-2 and max_abs(out.view(lq, heads, 128), ref) < 5e-2
    if kb is None:
        n_tiles = K.n_kv_tiles(rows)
        for splits in sorted({min(2, n_tiles), n_tiles}):
            po, pml = K.attention_workspace(splits, lq, heads, d)
            K.chunk_attention_partial(q.to(d), kd, vd, splits, po, pml)
            o2 = K.attention_merge(po, pml, splits, torch.empty_like(out))
            assert rel_l2(o2.view(lq, heads, 128), ref) < 1e-2


def test_chunk_attention_row_max_near_900(cuda_dev):
    """Real-weight hot heads reach row maxima of ~864 (the reference's const-max guard, model_fast.py:254-263):
    a key aligned with each query and scaled x80 sits in a late tile of a later chunk, so the running max jumps
    from ~4 to ~900 mid-window; the exact online softmax must still match fp32."""
    import lbw_b200.kernels as K
    g = _g(71)
    lq, heads, n = 160, 2, 700
    q = torch.randn(lq, heads, 128, generator=g).to(BF)
    ks = [torch.randn(n, heads, 128, generator=g) for _ in range(2)]
    for r in range(lq):                      # row r's hot key: 80 x q_r, in chunk 1 at position 300 + r
        ks[1][300 + r] = q[r].float() * 80.0
    ks = [k.to(BF) for k in ks]
    vs = [torch.randn(n, heads, 128, generator=g).to(BF) for _ in range(2)]
    d = cuda_dev
    logits = torch.einsum("qhd,khd->qhk", q.float(), torch.cat(ks).float()) / 128 ** 0.5
    assert float(logits.max()) > 800
    out = K.chunk_attention(q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs])
    ref = ob.attention(q, torch.cat(ks), torch.cat(vs))
    assert torch.isfinite(out).all()
    assert rel_l2(out.view(lq, heads, 128), ref) < 1e-2 and max_abs(out.view(lq, heads, 128), ref) < 5e-2


def test_chunk_attention_hot_head_rescale(cuda_dev):
    """Row maxima that grow by far more than 2^8 across KV tiles (hot heads, row max in the hundreds)."""
    import lbw_b200.kernels as K
    g = _g(7)
    lq, heads = 128, 1
    q = torch.randn(lq, heads, 128, generator=g).to(BF)
    k = torch.randn(1024, heads, 128, generator=g)
    k[512:] *= 6.0                          # later tiles have much larger scores
    k = k.to(BF)
    v = torch.randn(1024, heads, 128, generator=g).to(BF)
    out = K.chunk_attention(q.to(cuda_dev), [k.to(cuda_dev)], [v.to(cuda_dev)])
    ref = ob.attention(q, k, v)
    assert rel_l2(out.view(lq, heads, 128), ref) < 1e-2


def test_chunk_attention_key_bias(cuda_dev):
    import lbw_b200.kernels as K
    q, ks, vs = _attn_case(200, [96], 2, 9)
    bias = torch.zeros(96)
    bias[40:] = math.log(7.0)
    out = K.chunk_attention(q.to(cuda_dev), [ks[0].to(cuda_dev)], [vs[0].to(cuda_dev)], key_bias=bias.to(cuda_dev))
    ref = ob.attention(q, ks[0], vs[0], key_bias=bias)
    assert rel_l2(out.view(200, 2, 128), ref) < 1e-2


def test_cross_dedup_against_reference_golden(cuda_dev):
    from conftest import load_golden
    import lbw_b200.attention as A
    g = load_golden("cross_dedup")
    d = cuda_dev
    bias = A.cross_dedup_bias(g["ctx_k"].to(d), g["ctx_v"].to(d), g["kc"])
    assert torch.allclose(bias.cpu(), g["bias"])
    out = A.cross_attention_dedup(g["q"].unsqueeze(0).to(d), g["ctx_k"].to(d), g["ctx_v"].to(d), bias, g["kc"])
    assert rel_l2(out[0], g["out"]) < 1e-2 and rel_l2(out[0], g["full"]) < 1e-2


@pytest.mark.parametrize("c", [96, 1536, 5120, 6144])
@pytest.mark.parametrize("mode", ["mod", "affine", "mod_mx"])
def test_layernorm_mod(cuda_dev, mode, c):
    import lbw_b200.kernels as K
    g = _g(11)
    m = 257
    x = torch.randn(m, c, generator=g) * 2 + 0.5
    s, t = torch.randn(c, generator=g) * 0.1, torch.randn(c, generator=g) * 0.1
    out = torch.empty(m, c, dtype=BF, device=cuda_dev)
    ln = ob.layer_norm(x, 1e-6)
    if mode == "affine":
        K.layernorm_mod(x.to(cuda_dev), 1e-6, out, weight=s.to(cuda_dev), bias=t.to(cuda_dev))
        ref = ob.layer_norm(x, 1e-6, s, t).to(BF)
    else:
        K.layernorm_mod(x.to(cuda_dev), 1e-6, out, scale=s.to(cuda_dev), shift=t.to(cuda_dev), mx_qdq=mode == "mod_mx")
        ref = (ln * (1 + s) + t).to(BF)
        if mode == "mod_mx":
            ref = omx.qdq(ref)
    assert rel_l2(out, ref) < 2e-3


@pytest.mark.parametrize("grid,start,tok0,m,c", [((3, 4, 6), 6, 0, 72, 512), ((3, 30, 52), 18, 1170, 1170, 512),
                                                   ((3, 4, 6), 2, 12, 60, 5120), ((1, 2, 3), 0, 0, 6, 6144)])
def test_rmsnorm_rope(cuda_dev, grid, start, tok0, m, c):
    import lbw_b200.kernels as K
    import lbw_b200.rope as R
    g = _g(13)
    x = torch.randn(m, c, generator=g).to(BF)
    gamma = (1 + 0.02 * torch.randn(c, generator=g)).to(BF)
    ss = x.float().pow(2).sum(1)
    d = cuda_dev
    cos, sin = R.rope_tables(R.rope_freqs(), grid, start, d)
    out = torch.empty(m + 8, c, dtype=BF, device=d)
    K.rmsnorm_rope(x.to(d), ss.to(d), gamma.to(d), 1e-6, out, rope=(cos, sin, grid[0]), grid=grid, tok0=tok0,
                   out_row_off=8)
    gc, gs = ob.rope_grid(ob.rope_freqs(), grid, start)
    ref = ob.rope_apply(ob.rms_norm(x, gamma, 1e-6).view(m, c // 128, 128), gc[tok0:tok0 + m], gs[tok0:tok0 + m])
    assert rel_l2(out[8:].view(m, -1, 128), ref) < 2e-3


@pytest.mark.parametrize("grid,start,tok0,m,c", [((3, 4, 6), 6, 0, 72, 512), ((3, 30, 52), 18, 1170, 1170, 512),
                                                   ((3, 45, 80), 18, 3600, 2700, 5120)])
def test_rope_rotation_bits(cuda_dev, grid, start, tok0, m, c):
    """The kernel's rotation, in both RoPE modes, is bit-identical to the oracle's rotation of the kernel's own
    normalised rows (the same launch without RoPE): fp32 math, and the reference's bf16 mode (bf16 tables, every
    product and sum rounded to bf16; the oracle's bf16 rotation is pinned to the reference by rope_bf16.pt). The last
    case is a c4 shard: tokens 3,600.. of the 720p chunk, 40 heads."""
    import lbw_b200.kernels as K
    import lbw_b200.rope as R
    g = _g(23)
    d = cuda_dev
    x = torch.randn(m, c, generator=g).to(BF).to(d)
    gamma = (1 + 0.02 * torch.randn(c, generator=g)).to(BF).to(d)
    ss = x.float().pow(2).sum(1)
    cos, sin = R.rope_tables(R.rope_freqs(), grid, start, d)
    y = torch.empty(m, c, dtype=BF, device=d)
    K.rmsnorm_rope(x, ss, gamma, 1e-6, y)
    gc, gs = ob.rope_grid(ob.rope_freqs(), grid, start)
    for dt in (torch.float32, torch.bfloat16):
        out = torch.empty(m, c, dtype=BF, device=d)
        K.rmsnorm_rope(x, ss, gamma, 1e-6, out, rope=(cos, sin, grid[0]), grid=grid, tok0=tok0,
                       rope_bf16=dt == torch.bfloat16)
        ref = ob.rope_apply(y.cpu().view(m, c // 128, 128), gc[tok0:tok0 + m], gs[tok0:tok0 + m], dt)
        assert torch.equal(out.cpu().view(m, -1, 128), ref), dt


@pytest.mark.parametrize("grid,start,tok0,m,c", [((3, 4, 6), 6, 0, 72, 512), ((3, 30, 52), 18, 1170, 1170, 512)])
def test_qk_rmsnorm_rope_equals_two_launches(cuda_dev, grid, start, tok0, m, c):
    """The fused q + k launch gives the bits of the two separate rmsnorm_rope launches (own gammas, row sums and
    destinations; k written at a row offset into a wider chunk, as into the destination cache slot)."""
    import lbw_b200.kernels as K
    import lbw_b200.rope as R
    g = _g(19)
    d = cuda_dev
    q, k = torch.randn(m, c, generator=g).to(BF).to(d), torch.randn(m, c, generator=g).to(BF).to(d)
    gq, gk = [(1 + 0.02 * torch.randn(c, generator=g)).to(BF).to(d) for _ in range(2)]
    ssq, ssk = q.float().pow(2).sum(1), k.float().pow(2).sum(1)
    cos, sin = R.rope_tables(R.rope_freqs(), grid, start, d)
    rp = (cos, sin, grid[0])
    q1, k1 = torch.empty(m, c, dtype=BF, device=d), torch.full((m + 16, c), 3.0, dtype=BF, device=d)
    K.rmsnorm_rope(q, ssq, gq, 1e-6, q1, rope=rp, grid=grid, tok0=tok0)
    K.rmsnorm_rope(k, ssk, gk, 1e-6, k1, rope=rp, grid=grid, tok0=tok0, out_row_off=16)
    q2, k2 = torch.empty(m, c, dtype=BF, device=d), torch.full((m + 16, c), 3.0, dtype=BF, device=d)
    K.qk_rmsnorm_rope(q, ssq, gq, q2, k, ssk, gk, k2, 1e-6, rp, grid, tok0=tok0, k_row_off=16)
    assert torch.equal(q1, q2) and torch.equal(k1, k2)
    # the same with the reference's bf16 rotation
    K.rmsnorm_rope(q, ssq, gq, 1e-6, q1, rope=rp, grid=grid, tok0=tok0, rope_bf16=True)
    K.rmsnorm_rope(k, ssk, gk, 1e-6, k1, rope=rp, grid=grid, tok0=tok0, out_row_off=16, rope_bf16=True)
    K.qk_rmsnorm_rope(q, ssq, gq, q2, k, ssk, gk, k2, 1e-6, rp, grid, tok0=tok0, k_row_off=16, rope_bf16=True)
    assert torch.equal(q1, q2) and torch.equal(k1, k2)


def test_mx_quantize_bit_exact(cuda_dev):
    import lbw_b200.kernels as K
    g = _g(17)
    rows, k = 300, 512
    x = (torch.randn(rows, k, generator=g) * torch.logspace(-3, 3, rows).view(-1, 1)).to(BF)
    x[5] = 0
    x[7, :32] = 1000.0
    data, scales, deq = K.mx_quantize(x.to(cuda_dev), dequant=True)
    q, s = omx.quantize(x)
    assert torch.equal(data.cpu(), q.view(torch.uint8))
    assert torch.equal(scales.cpu(), omx.scales_tiled(s, k))
    assert torch.equal(deq.cpu().float(), omx.dequantize(q, s))


@pytest.mark.parametrize("splits", [1, 2, 3, 7])
def test_chunk_attention_split_kv_and_merge(cuda_dev, splits):
    import lbw_b200.kernels as K
    q, ks, vs = _attn_case(300, [200, 77, 500], 2, 19, qscale=2.0)
    d = cuda_dev
    kd, vd = [k.to(d) for k in ks], [v.to(d) for v in vs]
    po, pml = K.attention_workspace(splits + 1, 300, 2, d)
    K.chunk_attention_partial(q.to(d), kd, vd, splits, po, pml, slot0=1)
    out = torch.empty(300, 256, dtype=BF, device=d)
    K.attention_merge(po[1:], pml[1:], splits, out)
    ref = ob.attention(q, torch.cat(ks), torch.cat(vs))
    assert rel_l2(out.view(300, 2, 128), ref) < 1e-2
    # a cached-chunks call and a destination-chunk call merged = one call over the whole window
    K.chunk_attention_partial(q.to(d), kd[:-1], vd[:-1], 1, po, pml, slot0=0)
    K.chunk_attention_partial(q.to(d), kd[-1:], vd[-1:], 1, po, pml, slot0=1)
    out2 = torch.empty_like(out)
    K.attention_merge(po, pml, 2, out2)
    assert rel_l2(out2.view(300, 2, 128), ref) < 1e-2


@pytest.mark.parametrize("pieces", [0, 2, 3, 7])
def test_chunk_attention_tail_schedule(cuda_dev, pieces):
    """The tail schedule over 300 query rows x 75 heads = 150 windows (a window: one head's pair of 128-row query
    tiles against every key; here the second pair holds a lone 44-row tile): the windows of the full waves run
    whole and write exactly what lbw_chunk_attention writes; the windows past the last full wave (2 of them on
    148 SMs) are cut into `pieces` key ranges (0: the planned count) and merged, within fp32 rounding of the
    whole-window result (bf16 rounding of P) and against the fp32 oracle."""
    import lbw_b200.kernels as K
    d = cuda_dev
    heads, lq, rows = 75, 300, [200, 77, 500]
    q, ks, vs = _attn_case(lq, rows, heads, 41, qscale=2.0)
    qd, kd, vd = q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs]
    whole = K.chunk_attention(qd, kd, vd)
    n_tail, used = K.attention_tail_plan(lq, heads, rows, d, pieces)
    assert n_tail == 150 % torch.cuda.get_device_properties(d).multi_processor_count
    assert used == (pieces if pieces else used) and 1 < used <= 7
    out = K.chunk_attention_tail(qd, kd, vd, K.attention_tail_workspace(lq, heads, rows, d, pieces), pieces=pieces)
    torch.cuda.synchronize()
    n_dp = 150 - n_tail
    for w in range(150):
        head, pair = divmod(w, 2)
        r0, r1 = pair * 256, min(lq, pair * 256 + 256)
        got, want = out[r0:r1, head * 128:(head + 1) * 128], whole[r0:r1, head * 128:(head + 1) * 128]
        if w < n_dp:
            assert torch.equal(got, want), w
        else:
            # P is rounded to bf16 against each piece's own running max, so the rounding differs from the whole
            # window's (about 3e-3 of the output here)
            assert rel_l2(got, want) < 5e-3, (w, rel_l2(got, want))
            ref = ob.attention(q[r0:r1, head:head + 1], torch.cat(ks)[:, head:head + 1], torch.cat(vs)[:, head:head + 1])
            assert rel_l2(got.cpu().view(r1 - r0, 1, 128), ref) < 1e-2


def test_chunk_attention_tail_validation(cuda_dev):
    """More pieces than key tiles, and a workspace smaller than the plan, are refused before any launch."""
    import lbw_b200.kernels as K
    d = cuda_dev
    heads, lq, rows = 75, 300, [200, 77, 500]
    q, ks, vs = _attn_case(lq, rows, heads, 43)
    qd, kd, vd = q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs]
    with pytest.raises(ValueError, match="pieces"):
        K.attention_tail_plan(lq, heads, rows, d, 8)
    po, pml = K.attention_tail_workspace(lq, heads, rows, d, 3)
    with pytest.raises(ValueError, match="workspace blocks"):
        K.chunk_attention_tail(qd, kd, vd, (po[:1], pml[:1]), pieces=3)
    with pytest.raises(ValueError, match="workspace blocks"):
        K.chunk_attention_tail(qd, kd, vd, None, pieces=3)


def test_gated_attention_matches_ungated(cuda_dev):
    """With its gate already open, the gated kernel computes exactly what the ungated one does, in both output
    modes (direct and split-KV partials + merge); a gate chunk outside the window is rejected."""
    import lbw_b200.kernels as K
    d = cuda_dev
    q, ks, vs = _attn_case(300, [256, 200, 130], 2, 31)
    q, ks, vs = q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs]
    flag = torch.full((4,), 7, dtype=torch.int32, device=d)
    ref = K.chunk_attention(q, ks, vs)
    out = torch.empty_like(ref)
    K.chunk_attention_gated(q, ks, vs, flag.data_ptr(), 7, 2, out=out)
    assert torch.equal(out, ref)
    po, pml = K.attention_workspace(3, 300, 2, d)
    K.chunk_attention_partial(q, ks, vs, 3, po, pml)
    ref3 = K.attention_merge(po, pml, 3, torch.empty_like(ref))
    po2, pml2 = K.attention_workspace(3, 300, 2, d)
    K.chunk_attention_gated(q, ks, vs, flag.data_ptr(), 6, 1, n_splits=3, part_o=po2, part_ml=pml2)
    assert torch.equal(K.attention_merge(po2, pml2, 3, torch.empty_like(ref)), ref3)
    # the tail schedule (here every window is cut: 4 windows), gated and ungated
    wst = K.attention_tail_workspace(300, 2, [256, 200, 130], d, 3)
    reft = K.chunk_attention_tail(q, ks, vs, wst, pieces=3)
    outt = K.chunk_attention_tail(q, ks, vs, wst, pieces=3, gate_flag_ptr=flag.data_ptr(), gate_value=7, gate_chunk=2)
    assert torch.equal(outt, reft)
    assert rel_l2(reft, ref) < 5e-3
    with pytest.raises(ValueError, match="gate chunk"):
        K.chunk_attention_gated(q, ks, vs, flag.data_ptr(), 7, 3, out=out)


def test_gated_attention_times_out_on_a_gate_that_never_opens(cuda_dev, monkeypatch):
    """A gate word that nothing ever raises: every CTA's bounded gate wait (LBW_GATE_TIMEOUT_S, set to one second
    here; 120 s by default) runs out, the kernel drains its copies and MMAs and returns, and the host reads the
    timeout (0x100 | 0x23, the gate site) from the device status word; the context stays usable for the next
    launch. One wave of CTAs (2 heads x one 256-row query block), so the wait is paid once."""
    import time
    import lbw_b200._lib as L
    import lbw_b200.kernels as K
    monkeypatch.setenv("LBW_GATE_TIMEOUT_S", "1")
    d = cuda_dev
    q, ks, vs = _attn_case(256, [256, 200], 2, 37)
    q, ks, vs = q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs]
    flag = torch.zeros(4, dtype=torch.int32, device=d)       # stays 0; the kernel waits for 1
    out = torch.zeros(256, 256, dtype=BF, device=d)
    torch.cuda.synchronize()
    t0 = time.monotonic()
    K.chunk_attention_gated(q, ks, vs, flag.data_ptr(), 1, 1, out=out)
    with pytest.raises(L.LbwError, match="0x123"):
        L.check_device_status()
    assert 0.9 < time.monotonic() - t0 < 30
    assert L.check_device_status() == 0                      # read and cleared
    ref = K.chunk_attention(q, ks, vs)                       # the context still runs kernels
    torch.cuda.synchronize()
    assert rel_l2(ref.view(256, 2, 128), ob.attention(q.cpu(), torch.cat(ks).cpu(), torch.cat(vs).cpu())) < 1e-2


def test_split_count_is_validated(cuda_dev):
    import lbw_b200.kernels as K
    q, ks, vs = _attn_case(128, [100], 1, 23)
    po, pml = K.attention_workspace(2, 128, 1, cuda_dev)
    with pytest.raises(ValueError, match="KV splits"):
        K.chunk_attention_partial(q.to(cuda_dev), [ks[0].to(cuda_dev)], [vs[0].to(cuda_dev)], 2, po, pml)


def test_small_m_residual_and_qkv_use_narrow_tiles(cuda_dev):
    """M = 1350 rows (one of 8 ranks at 720p): 256-wide tiles would fill 1.5 waves, so 128-wide ones run."""
    import lbw_b200.kernels as K
    g = _g(29)
    m, c = 1350, 1536
    h = torch.randn(m, c, generator=g).to(BF)
    w = (torch.randn(3 * c, c, generator=g) * 0.02).to(BF)
    b = (torch.randn(3 * c, generator=g) * 0.02).to(BF)
    d = cuda_dev
    q, k = torch.empty(m, c, dtype=BF, device=d), torch.empty(m, c, dtype=BF, device=d)
    ss = torch.empty(2, m, device=d)
    v = torch.empty(m, c, dtype=BF, device=d)
    K.qkv_proj(h.to(d), w.to(d), b.to(d), q, k, ss[0], ss[1], v)
    ref = ob.linear(h, w, b)
    assert rel_l2(q, ref[:, :c]) < 4e-3 and rel_l2(v, ref[:, 2 * c:]) < 4e-3
    assert rel_l2(ss[1], k.float().pow(2).sum(1)) < 1e-5
    x = torch.randn(m, 5120, generator=g)
    wo = (torch.randn(5120, c, generator=g) * 0.02).to(BF)
    xd = x.to(d)
    K.linear_residual(h.to(d), wo.to(d), None, xd)
    assert rel_l2(xd - x.to(d), ob.linear(h, wo, None).float()) < 5e-3


def test_device_init_destroy(cuda_dev):
    """lbw_init makes the per-device state up front (idempotent, a missing device is a ValueError, the caller's
    device stays current); lbw_destroy releases it after the device is idle, and the next call recreates it:
    the same attention before and after gives the same bits and a clean status."""
    import lbw_b200._lib as L
    import lbw_b200.kernels as K
    d = cuda_dev
    L.init_device(d)
    L.init_device(d)
    with pytest.raises(ValueError):
        L.init_device(torch.device("cuda", 63))
    assert torch.cuda.current_device() == d.index
    q, ks, vs = _attn_case(200, [256, 130], 2, 41)
    q, ks, vs = q.to(d), [k.to(d) for k in ks], [v.to(d) for v in vs]
    ref = K.chunk_attention(q, ks, vs)
    assert L.check_device_status() == 0
    L.destroy_device(d)
    assert torch.cuda.current_device() == d.index
    assert L.check_device_status() == 0          # no status word now: nothing to read, nothing allocated
    out = K.chunk_attention(q, ks, vs)           # recreates the status word
    assert torch.equal(out, ref)
    assert L.check_device_status() == 0
