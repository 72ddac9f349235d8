"""The kernels as torch.ops.lbw.* operators and the block under torch.compile, plus kv_write=False.

The reference compiles groups of blocks with torch.compile(fullgraph=True) (wan/modules/model_fast.py:3808-3826);
the drop-in block must trace into one graph through the registered operators (lbw_b200.ops) and give the eager
result. kv_write=False (LINGBOT_STEP_NOWRITE, model_fast.py:2135-2143, :3821-3835) attends the new chunk without
writing the destination cache slot."""
import pytest
import torch

from conftest import rel_l2
from oracle.inputs import BlockCase, make_case

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _block(case, p, dev):
    import lbw_b200.block as B
    blk = B.CausalWanAttentionBlock(case.dim, case.ffn, case.heads, qk_norm=True, cross_attn_norm=True, ffn_mx=True)
    sd = blk.state_dict()
    for k, v in p.items():
        sd[k] = v.to(sd[k].dtype)
    blk.load_state_dict(sd)
    return blk.to(dev)


def _inputs(case, inp, dev):
    C, H, Lq = case.dim, case.heads, case.lq
    ks = [k.unsqueeze(0).to(dev) for k in inp["k_lead"]] + [torch.zeros(1, Lq, H, 128, dtype=BF, device=dev)]
    vs = [v.unsqueeze(0).to(dev) for v in inp["v_lead"]] + [torch.zeros(1, Lq, H, 128, dtype=BF, device=dev)]
    cc = {"k": torch.zeros(1, case.text_len, H, 128, dtype=BF, device=dev),
          "v": torch.zeros(1, case.text_len, H, 128, dtype=BF, device=dev), "is_init": torch.zeros(1, device=dev)}
    film = (inp["film"][0].unsqueeze(0).to(dev), inp["film"][1].unsqueeze(0).to(dev))
    return ks, vs, cc, film


def test_ops_registered():
    import lbw_b200.ops as O
    for name in O.OPS:
        assert hasattr(torch.ops.lbw, name), name


def test_block_under_torch_compile_fullgraph(cuda_dev):
    """torch.compile(fullgraph=True) of the block forward (aot_eager: the traced graph runs the operators, no code
    generation) equals the eager forward, on the second call too (the destination chunk is rewritten)."""
    case = BlockCase(dim=256, ffn=512, grid=(3, 4, 6), n_lead=2, text_len=32, start_frame=6, seed=51)
    p, inp = make_case(case)
    d = cuda_dev
    blk = _block(case, p, d)
    ks, vs, cc, film = _inputs(case, inp, d)
    C = case.dim
    f, h, w = case.grid
    x = inp["x"].unsqueeze(0).to(d)
    e = inp["e0"].view(1, 1, 6, C).to(d)
    ctx = inp["context"].unsqueeze(0).to(d)

    def fwd(x, e, ks, vs):
        return blk(x, e, grid_ints=[case.grid], context=ctx, crossattn_cache=cc, current_start=case.start_frame * h * w,
                   frame_seqlen=h * w, kv_chunks=(ks, vs), dit_cond_dict={"cam_film": film}, cross_attn_first_call=False)

    blk(x, e, grid_ints=[case.grid], context=ctx, crossattn_cache=cc, current_start=case.start_frame * h * w,
        frame_seqlen=h * w, kv_chunks=(ks, vs), dit_cond_dict={"cam_film": film}, cross_attn_first_call=True)
    ref = fwd(x, e, ks, vs)
    k_ref = ks[-1].clone()
    torch._dynamo.reset()
    cfwd = torch.compile(fwd, fullgraph=True, backend="aot_eager")
    for _ in range(2):
        ks[-1].zero_()
        got = cfwd(x, e, ks, vs)
        torch.cuda.synchronize()
        assert torch.equal(ks[-1], k_ref)
        assert rel_l2(got, ref) < 1e-6


def test_kv_write_false_leaves_the_slot(cuda_dev):
    case = BlockCase(dim=256, ffn=512, grid=(3, 4, 6), n_lead=2, text_len=32, start_frame=6, seed=53)
    p, inp = make_case(case)
    d = cuda_dev
    blk = _block(case, p, d)
    ks, vs, cc, film = _inputs(case, inp, d)
    C = case.dim
    f, h, w = case.grid
    kw = dict(grid_ints=[case.grid], context=inp["context"].unsqueeze(0).to(d), crossattn_cache=cc,
              current_start=case.start_frame * h * w, frame_seqlen=h * w, dit_cond_dict={"cam_film": film})
    x = inp["x"].unsqueeze(0).to(d)
    e = inp["e0"].view(1, 1, 6, C).to(d)
    ref = blk(x, e, kv_chunks=(ks, vs), cross_attn_first_call=True, **kw)
    k_new, v_new = ks[-1].clone(), vs[-1].clone()
    ks[-1].fill_(0.5)
    vs[-1].fill_(-0.25)
    got = blk(x, e, kv_chunks=(ks, vs), cross_attn_first_call=False, kv_write=False, **kw)
    torch.cuda.synchronize()
    assert torch.all(ks[-1] == 0.5) and torch.all(vs[-1] == -0.25)        # the slot is untouched
    assert torch.equal(got, ref)                                          # the same K/V were attended
    ws = blk._ws.new_kv(case.lq)
    assert torch.equal(ws[0].view_as(k_new), k_new) and torch.equal(ws[1].view_as(v_new), v_new)


def _opcheck_cases(d):
    import lbw_b200.kernels as K
    g = torch.Generator(device=d).manual_seed(61)
    r = lambda *s, dt=torch.float32, std=1.0: (torch.randn(*s, generator=g, device=d) * std).to(dt)  # noqa: E731
    m, c, n = 200, 512, 256
    ops = torch.ops.lbw
    x = r(m, c)
    a, w, b = r(m, c, dt=BF), r(n, c, dt=BF, std=0.05), r(n, dt=BF, std=0.05)
    q, k, v = r(m, 2, 128, dt=BF), r(300, 2, 128, dt=BF), r(300, 2, 128, dt=BF)
    wd, ws, _ = K.mx_quantize(w)
    ad, as_, _ = K.mx_quantize(a)
    import lbw_b200.rope as R
    rope = R.rope_tables(R.rope_freqs(), (9, 4, 6), 6, d)   # a 216-token grid holds the m = 200 rows
    cases = {
        "layernorm_mod": (ops.layernorm_mod, (x, 1e-6, torch.empty(m, c, dtype=BF, device=d), r(c, std=0.1),
                                              r(c, std=0.1), None, None, False)),
        "linear_residual": (ops.linear_residual, (a, w, b, r(m, n), r(n, std=0.1), r(m, n, dt=BF, std=0.1),
                                                  r(m, n, dt=BF, std=0.1))),
        "linear_rowss": (ops.linear_rowss, (a, w, b, torch.empty(m, n, dtype=BF, device=d),
                                            torch.zeros(m, device=d))),
        "chunk_attention": (ops.chunk_attention, (q, [k], [v], None, 128 ** -0.5,
                                                  torch.empty(m, 256, dtype=BF, device=d))),
        "chunk_attention_tail": (ops.chunk_attention_tail, (q, [k], [v], None, 128 ** -0.5,
                                                            torch.empty(m, 256, dtype=BF, device=d),
                                                            *K.attention_tail_workspace(m, 2, [300], d, 3), 3)),
        "rmsnorm_rope": (ops.rmsnorm_rope, (a, (a.float() ** 2).sum(1), r(c, dt=BF), 1e-6,
                                            torch.empty(m, c, dtype=BF, device=d), None, None, 0, 0, 0, 0, 0, False)),
        "qk_rmsnorm_rope": (ops.qk_rmsnorm_rope, (a, (a.float() ** 2).sum(1), r(c, dt=BF),
                                                  torch.empty(m, c, dtype=BF, device=d), a.flip(0).contiguous(),
                                                  (a.float() ** 2).sum(1).flip(0).contiguous(), r(c, dt=BF),
                                                  torch.empty(m + 8, c, dtype=BF, device=d), 1e-6, *rope,
                                                  9, 4, 6, 0, 0, 8, True)),
        "mx_quantize": (ops.mx_quantize, (a, "e4m3")),
        "mx_quantize_into": (ops.mx_quantize_into, (a, torch.empty_like(ad), torch.empty_like(as_), "e4m3")),
        "mx_linear": (ops.mx_linear, (ad, as_, wd, ws, b, "e4m3")),
    }
    return cases


@pytest.mark.parametrize("name", ["layernorm_mod", "linear_residual", "linear_rowss", "chunk_attention",
                                  "chunk_attention_tail", "rmsnorm_rope", "qk_rmsnorm_rope", "mx_quantize", "mx_quantize_into",
                                  "mx_linear"])
def test_opcheck(cuda_dev, name):
    """torch.library.opcheck: each operator's schema (the tensors it declares it writes are the ones it writes, new
    outputs are new), its fake implementation (same output metadata as the real kernel) and its behaviour under
    compilation with dynamic shapes."""
    op, args = _opcheck_cases(cuda_dev)[name]
    res = torch.library.opcheck(op, args, test_utils=("test_schema", "test_faketensor", "test_aot_dispatch_dynamic"),
                                raise_exception=False)
    assert all(v == "SUCCESS" for v in res.values()), res
