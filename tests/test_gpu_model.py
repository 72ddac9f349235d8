"""The whole causal-fast model forward (CausalWanModel: patch/camera/text/timestep embeddings, the blocks on
the chunked KV cache, head, unpatchify) against the reference's own WanModelFast.forward on the same seeded
inputs (tests/golden/model_forward.pt)."""
import pytest
import torch

from conftest import load_golden, max_abs, rel_l2
from oracle.inputs import ModelCase, make_model_case

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _build(case, dev):
    import lbw_b200.model as M
    m = M.CausalWanModel(model_type="i2v", patch_size=(1, 2, 2), text_len=case.text_len, in_dim=case.in_dim,
                         dim=case.dim, ffn_dim=case.ffn, freq_dim=case.freq_dim, text_dim=case.text_dim,
                         out_dim=case.out_dim, num_heads=case.heads, num_layers=case.layers, ffn_mx=False)
    sd, inp = make_model_case(case)
    msd = m.state_dict()
    for k, v in sd.items():
        msd[k] = v.to(msd[k].dtype)
    m.load_state_dict(msd)
    return m.to(dev), inp


def _cache(case, inp, dev):
    import lbw_b200.chunked_kv_cache as ckv
    L, H = case.lq, case.heads
    cache = ckv.allocate_self_kv_chunks(case.layers, 1, L, H, 128, case.n_chunks, BF, dev)
    for bc, lead in zip(cache, inp["cache"]):
        for slot, (k, v) in enumerate(lead):
            bc["k"][slot].copy_(k.unsqueeze(0))
            bc["v"][slot].copy_(v.unsqueeze(0))
    cc = [{"k": torch.zeros(1, case.text_len, H, 128, dtype=BF, device=dev),
           "v": torch.zeros(1, case.text_len, H, 128, dtype=BF, device=dev), "is_init": torch.zeros(1, device=dev)}
          for _ in range(case.layers)]
    return cache, cc


def _run(m, case, inp, cache, cc, dev, skip_head=False):
    L = case.lq
    return m([inp["x"].to(dev)], inp["t"].to(dev), [inp["context"].to(dev)], L, y=[inp["y"].to(dev)],
             dit_cond_dict={"c2ws_plucker_emb": [inp["cam"].to(dev)]}, kv_cache=cache, crossattn_cache=cc,
             current_start=case.chunk_index * L, frame_seqlen=L // case.grid[0], cross_attn_first_call=True,
             skip_head=skip_head)


def test_model_forward_vs_reference_golden(cuda_dev):
    g = load_golden("model_forward")
    case = ModelCase(**g["case"])
    m, inp = _build(case, cuda_dev)
    cache, cc = _cache(case, inp, cuda_dev)
    out = _run(m, case, inp, cache, cc, cuda_dev)
    torch.cuda.synchronize()
    o = out[0].float().cpu()
    assert o.shape == g["out"].shape
    assert rel_l2(o, g["out"]) < 1e-2 and max_abs(o, g["out"]) < 5e-2
    dest = g["dest"]
    for i in range(case.layers):
        assert rel_l2(cache[i]["k"][dest][0].cpu(), g["k_dest"][i]) < 1e-2
        assert rel_l2(cache[i]["v"][dest][0].cpu(), g["v_dest"][i]) < 1e-2
        assert rel_l2(cc[i]["k"][0].cpu(), g["ctx_k"][i]) < 1e-2


def test_model_kv_commit_forward_writes_the_cache(cuda_dev):
    """skip_head (the KV-commit forward at t = 0 in the reference) returns None but writes the same K/V."""
    g = load_golden("model_forward")
    case = ModelCase(**g["case"])
    m, inp = _build(case, cuda_dev)
    cache, cc = _cache(case, inp, cuda_dev)
    assert _run(m, case, inp, cache, cc, cuda_dev, skip_head=True) is None
    torch.cuda.synchronize()
    for i in range(case.layers):
        assert rel_l2(cache[i]["k"][g["dest"]][0].cpu(), g["k_dest"][i]) < 1e-2


def test_model_from_checkpoint_folder_vs_reference_golden(cuda_dev, tmp_path):
    """The reference-layout checkpoint folder (config.json + sharded safetensors) through load_model gives the
    golden forward."""
    import lbw_b200.checkpoint as ck
    from test_host import _write_checkpoint
    g = load_golden("model_forward")
    case, _ = _write_checkpoint(tmp_path, sharded=True)
    m, unexpected = ck.load_model(str(tmp_path), device=cuda_dev)
    assert unexpected == []
    _, inp = make_model_case(case)
    cache, cc = _cache(case, inp, cuda_dev)
    o = _run(m, case, inp, cache, cc, cuda_dev)[0].float().cpu()
    assert rel_l2(o, g["out"]) < 1e-2 and max_abs(o, g["out"]) < 5e-2


def test_forward_fused_equals_commit_then_step(cuda_dev):
    """forward_fused (LINGBOT_FUSE_COMMIT's signature): chunk a's commit at t = 0, then chunk b's step, with the
    same output and cache as the two forwards called one after the other."""
    g = load_golden("model_forward")
    case = ModelCase(**g["case"])
    m, inp = _build(case, cuda_dev)
    d, L = cuda_dev, case.lq
    fs = L // case.grid[0]
    xb = (inp["x"] * 0.5).to(d)
    tb = torch.tensor([700.0], device=d)
    ca, cb = [inp["cam"].to(d)], [(inp["cam"] * 0.9).to(d)]
    a, b = case.chunk_index, case.chunk_index + 1
    cache1, cc1 = _cache(case, inp, d)
    cache2, cc2 = _cache(case, inp, d)
    for cc in (cc1, cc2):   # the cross cache is filled by an earlier forward, as in the reference
        m([inp["x"].to(d)], inp["t"].to(d), [inp["context"].to(d)], L, y=[inp["y"].to(d)],
          kv_cache=_cache(case, inp, d)[0], crossattn_cache=cc, current_start=a * L, frame_seqlen=fs,
          cross_attn_first_call=True, skip_head=True)
    zero = torch.zeros(1, device=d)
    out = m.forward_fused(inp["x"].to(d), inp["y"].to(d), ca, zero, 0.0, a, xb, inp["y"].to(d), cb, tb, 700.0, b,
                          context=[inp["context"].to(d)], seq_len=L, kv_cache=cache1, crossattn_cache=cc1,
                          frame_seqlen=fs)
    assert m([inp["x"].to(d)], zero, [inp["context"].to(d)], L, y=[inp["y"].to(d)],
             dit_cond_dict={"c2ws_plucker_emb": ca}, kv_cache=cache2, crossattn_cache=cc2, current_start=a * L,
             frame_seqlen=fs, cross_attn_first_call=False, skip_head=True) is None
    ref = m([xb], tb, [inp["context"].to(d)], L, y=[inp["y"].to(d)], dit_cond_dict={"c2ws_plucker_emb": cb},
            kv_cache=cache2, crossattn_cache=cc2, current_start=b * L, frame_seqlen=fs, cross_attn_first_call=False)
    torch.cuda.synchronize()
    assert torch.equal(out[0], ref[0]) and torch.isfinite(out[0]).all()
    for i in range(case.layers):
        for key in ("k", "v"):
            for s1, s2 in zip(cache1[i][key], cache2[i][key]):
                assert torch.equal(s1, s2)
