"""Generate golden fixtures from the REFERENCE implementation's own PyTorch code.

Run where a checkout of the reference exists, naming it in $LBW_REFERENCE:
    LBW_REFERENCE=<reference checkout> python tests/golden/make_golden.py

It imports yahavb/lingbot-world-v2's wan/modules/model_fast.py on CPU through small import shims
(the Neuron-only packages diffusers/easydict/torch_neuronx are absent here), builds one
CausalWanAttentionBlock (model_fast.py:2837-3116) with the seeded parameters of oracle.inputs,
runs its chunked-KV forward (kv_chunks path, exact attention -> SDPA) and saves the block output,
the destination-chunk K/V it writes and the outputs of self_attn / cross_attn / ffn. It also saves
the reference's cross_dedup_bias + cross_attention_dedup (wan/modules/attention.py:516-554) on a
duplicated-context case, the reference's RoPE grids, its camera FiLM MLP, and one whole
WanModelFast.forward (model_fast.py:3283-3935) of a 2-block i2v model with the camera condition, and the
Wan 2.1 VAE decode (wan/modules/vae2_1.py) of a small latent, and the RoPE rotation in the reference's bf16 mode
(`make_golden.py rope_bf16` writes that fixture alone). Inputs are NOT stored (except the small VAE latent and the
RoPE rows): they are regenerated from the seed by oracle.inputs / oracle.vae; a checksum guards against drift.

Nothing at test or bench time reads the reference; only the .pt files produced here are used.
"""
import contextlib
import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("LBW_REFERENCE", "")
sys.path.insert(0, ROOT)

from oracle.inputs import BlockCase, ModelCase, make_case, make_model_case  # noqa: E402

CASES = {
    "block_flat": BlockCase(dim=256, ffn=512, grid=(3, 4, 6), n_lead=2, text_len=32, start_frame=6, seed=1),
    "block_peaked": BlockCase(dim=256, ffn=384, grid=(3, 5, 7), lead_rows=(50, 105), text_len=40, start_frame=9,
                              peaked=True, seed=2),
    "block_nofilm": BlockCase(dim=384, ffn=512, grid=(2, 4, 8), n_lead=1, text_len=24, start_frame=2, film=False,
                              seed=3),
}
DEDUP = BlockCase(dim=256, ffn=256, grid=(1, 8, 8), n_lead=0, text_len=64, dedup_rows=20, peaked=True, seed=4)
CAM = BlockCase(dim=256, ffn=256, grid=(1, 6, 8), n_lead=0, text_len=16, cam=True, seed=6)
MODEL = ModelCase()


def install_shims():
    """Minimal stand-ins for the Neuron-only imports of the reference modules."""
    d = types.ModuleType("diffusers")
    cu = types.ModuleType("diffusers.configuration_utils")
    mu = types.ModuleType("diffusers.models.modeling_utils")
    dm = types.ModuleType("diffusers.models")

    class ConfigMixin:
        pass

    def register_to_config(f):
        return f

    cu.ConfigMixin, cu.register_to_config = ConfigMixin, register_to_config
    mu.ModelMixin = torch.nn.Module
    d.configuration_utils, d.models, dm.modeling_utils = cu, dm, mu
    sys.modules.update({"diffusers": d, "diffusers.configuration_utils": cu, "diffusers.models": dm,
                        "diffusers.models.modeling_utils": mu})
    ed = types.ModuleType("easydict")

    class EasyDict(dict):
        __getattr__ = dict.get

    ed.EasyDict = EasyDict
    sys.modules["easydict"] = ed
    # packages without their __init__ (wan/__init__.py pulls the whole pipeline)
    for name, sub in (("wan", ""), ("wan.modules", "modules"), ("wan.distributed", "distributed")):
        m = types.ModuleType(name)
        m.__path__ = [os.path.join(REF, "wan", sub) if sub else os.path.join(REF, "wan")]
        sys.modules[name] = m
    sys.path.insert(0, REF)
    # model_fast decorates with torch.compile(backend="neuron") at import
    from torch._dynamo import register_backend

    @register_backend(name="neuron")
    def _neuron_backend(gm, example_inputs):
        return gm.forward

    # autocast('neuron', ...) -> the CPU autocast (fp32 requests are a no-op there)
    orig = torch.amp.autocast

    class _Autocast(orig):
        def __init__(self, device_type, *a, **k):
            super().__init__("cpu" if device_type == "neuron" else device_type, *a, **k)

    torch.amp.autocast = _Autocast


def checksum(p, inp):
    s = 0.0
    for t in list(p.values()) + [inp["x"], inp["e0"], inp["context"]] + inp["k_lead"] + inp["v_lead"]:
        s += float(t.float().abs().sum())
    return s


def run_block(mf, case):
    p, inp = make_case(case)
    C, H, (f, h, w) = case.dim, case.heads, case.grid
    Lq = case.lq
    blk = mf.CausalWanAttentionBlock(C, case.ffn, H, local_attn_size=-1, sink_size=0, qk_norm=True,
                                     cross_attn_norm=True, eps=1e-6)
    blk = blk.to(torch.bfloat16)
    blk.modulation.data = blk.modulation.data.float()
    blk.norm3.weight.data = blk.norm3.weight.data.float()
    blk.norm3.bias.data = blk.norm3.bias.data.float()
    sd = blk.state_dict()
    for k_, v_ in p.items():
        assert k_ in sd, k_
        sd[k_] = v_.to(sd[k_].dtype)
    blk.load_state_dict(sd)
    blk.eval()
    caps = {}
    for nm in ("self_attn", "cross_attn", "ffn"):
        getattr(blk, nm).register_forward_hook(lambda m, a, o, nm=nm: caps.__setitem__(nm, o.detach().clone()))
    d = 128
    freqs = torch.cat([mf.rope_params(1024, d - 4 * (d // 6)), mf.rope_params(1024, 2 * (d // 6)),
                       mf.rope_params(1024, 2 * (d // 6))], dim=1)
    grid_sizes = torch.tensor([[f, h, w]])
    cos_g, sin_g = mf._causal_rope_grids_build(freqs, grid_sizes, "cpu", case.start_frame)
    k_chunks = [k.unsqueeze(0).clone() for k in inp["k_lead"]] + [torch.zeros(1, Lq, H, d, dtype=torch.bfloat16)]
    v_chunks = [v.unsqueeze(0).clone() for v in inp["v_lead"]] + [torch.zeros(1, Lq, H, d, dtype=torch.bfloat16)]
    ccache = {"k": torch.zeros(1, case.text_len, H, d, dtype=torch.bfloat16),
              "v": torch.zeros(1, case.text_len, H, d, dtype=torch.bfloat16), "is_init": torch.zeros(1)}
    cond = {"cam_film": (inp["film"][0].unsqueeze(0), inp["film"][1].unsqueeze(0))} if inp["film"] else None
    with torch.no_grad():
        out = blk(inp["x"].unsqueeze(0), inp["e0"].view(1, 1, 6, C), seq_lens=torch.tensor([Lq]),
                  grid_sizes=grid_sizes, freqs=freqs, context=inp["context"].unsqueeze(0), context_lens=None,
                  dit_cond_dict=cond, crossattn_cache=ccache, current_start=case.start_frame * h * w,
                  frame_seqlen=h * w, cross_attn_first_call=True, rope_grids=(cos_g, sin_g),
                  rope_local_grid=[(f, h, w)], kv_chunks=(k_chunks, v_chunks), grid_ints=[(f, h, w)])
    return dict(case=case.__dict__, checksum=checksum(p, inp), x=out[0].float(), k_dest=k_chunks[-1][0].clone(),
                v_dest=v_chunks[-1][0].clone(), self_attn=caps["self_attn"][0], cross_attn=caps["cross_attn"][0],
                ffn=caps["ffn"][0], ctx_k=ccache["k"][0].clone(), ctx_v=ccache["v"][0].clone(),
                rope_cos=cos_g[0].reshape(Lq, -1).clone(), rope_sin=sin_g[0].reshape(Lq, -1).clone())


def run_dedup(attn_mod, mf):
    """Reference cross_dedup on a context whose rows >= dedup_rows are identical."""
    case = DEDUP
    p, inp = make_case(case)
    C, H, d = case.dim, case.heads, 128
    from oracle.block import cross_kv
    ck, cv = cross_kv(p, inp["context"])            # [T, H, d] each (restated projection)
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, case.lq, H, d, generator=g).to(torch.bfloat16)
    kc = 32
    bias = attn_mod.cross_dedup_bias(ck, cv, kc)
    out = attn_mod.cross_attention_dedup(q, ck.permute(1, 2, 0).contiguous(), cv.permute(1, 0, 2).contiguous(),
                                         bias, kc)
    full = attn_mod.attention(q, ck.unsqueeze(0), cv.unsqueeze(0))
    return dict(case=case.__dict__, q=q[0], ctx_k=ck, ctx_v=cv, kc=kc, bias=bias, out=out[0], full=full[0])


def run_cam(mf):
    """Reference CausalWanAttentionBlock.cam_film (model_fast.py:2882-2891) on a seeded camera condition."""
    case = CAM
    p, inp = make_case(case)
    blk = mf.CausalWanAttentionBlock(case.dim, case.ffn, case.heads, qk_norm=True, cross_attn_norm=True, eps=1e-6)
    blk = blk.to(torch.bfloat16)
    sd = blk.state_dict()
    for k_, v_ in p.items():
        sd[k_] = v_.to(sd[k_].dtype)
    blk.load_state_dict(sd)
    with torch.no_grad():
        scale, shift = blk.cam_film(inp["cam"].unsqueeze(0))
    return dict(case=case.__dict__, checksum=checksum(p, inp), scale=scale[0].clone(), shift=shift[0].clone())


def run_model(mf, ckv):
    """Reference WanModelFast.forward (model_fast.py:3283-3935) on the chunked cache, i2v with the camera
    condition: patch + camera + text + timestep embeddings, the blocks, the head and unpatchify."""
    case = MODEL
    sd, inp = make_model_case(case)
    m = mf.WanModelFast(model_type="i2v", patch_size=(1, 2, 2), text_len=case.text_len, in_dim=case.in_dim,
                        dim=case.dim, ffn_dim=case.ffn, freq_dim=case.freq_dim, text_dim=case.text_dim,
                        out_dim=case.out_dim, num_heads=case.heads, num_layers=case.layers, qk_norm=True,
                        cross_attn_norm=True, eps=1e-6)
    m = m.to(torch.bfloat16)
    for name in ("time_embedding", "time_projection", "head"):   # fp32 under the reference's fp32 autocast
        getattr(m, name).float()
    for blk in m.blocks:
        blk.modulation.data = blk.modulation.data.float()
        blk.norm3.float()
    msd = m.state_dict()
    for k_, v_ in sd.items():
        assert k_ in msd, k_
        msd[k_] = v_.to(msd[k_].dtype)
    missing = [k_ for k_ in msd if k_ not in sd and not k_.endswith("freqs")]
    assert not missing, missing
    m.load_state_dict(msd)
    m.eval()
    L, H = case.lq, case.heads
    cache = ckv.allocate_self_kv_chunks(case.layers, 1, L, H, 128, case.n_chunks, torch.bfloat16, "cpu")
    for bc, lead in zip(cache, inp["cache"]):
        for slot, (k_, v_) in enumerate(lead):
            bc["k"][slot].copy_(k_.unsqueeze(0))
            bc["v"][slot].copy_(v_.unsqueeze(0))
    cc = [{"k": torch.zeros(1, case.text_len, H, 128, dtype=torch.bfloat16),
           "v": torch.zeros(1, case.text_len, H, 128, dtype=torch.bfloat16), "is_init": torch.zeros(1)}
          for _ in range(case.layers)]
    caps = {}
    m.head.register_forward_hook(lambda mod, a, o: caps.__setitem__("head", o.detach().float().clone()))
    m.text_embedding.register_forward_hook(lambda mod, a, o: caps.__setitem__("context", o.detach().clone()))
    f = case.grid[0]
    with torch.no_grad():
        out = m([inp["x"]], inp["t"], [inp["context"]], L, y=[inp["y"]],
                dit_cond_dict={"c2ws_plucker_emb": [inp["cam"]]}, kv_cache=cache, crossattn_cache=cc,
                current_start=case.chunk_index * L, frame_seqlen=L // f, cross_attn_first_call=True)
    dest, lead_slots = ckv.chunk_routing(case.chunk_index, case.n_chunks)
    return dict(case=case.__dict__, out=out[0].float().clone(), head=caps["head"][0], context=caps["context"][0],
                dest=dest, leading=tuple(lead_slots),
                k_dest=[bc["k"][dest][0].clone() for bc in cache], v_dest=[bc["v"][dest][0].clone() for bc in cache],
                ctx_k=[c["k"][0].clone() for c in cc], ctx_v=[c["v"][0].clone() for c in cc])


VAE_CFG = dict(dim=32)          # the Wan 2.1 decoder structure (dim_mult 1,2,4,4, 2 res blocks, temporal x4) at dim 32
VAE_SEED = 5


def run_vae():
    """The reference's WanVAE_.decode (wan/modules/vae2_1.py:548-572) and decode_chunk over two calls (:574-596)
    of a 3-frame 4x6 latent, with oracle.vae's seeded parameters, and the bf16 latent scale of Wan2_1_VAE."""
    from oracle import vae as ov
    with contextlib.redirect_stdout(sys.stderr):
        import wan.modules.vae2_1 as v21
    m = v21.WanVAE_(dim=VAE_CFG["dim"], z_dim=16, dim_mult=[1, 2, 4, 4], num_res_blocks=2, attn_scales=[],
                    temperal_downsample=[False, True, True]).eval()
    params = ov.make_params(VAE_SEED, **VAE_CFG)
    sd = m.state_dict()
    names = {k for k in sd if k.startswith("conv2.") or k.startswith("decoder.")}
    assert names == set(params), sorted(names ^ set(params))[:5]
    for k, v in params.items():
        assert tuple(sd[k].shape) == tuple(v.shape), k
        sd[k] = v
    m.load_state_dict(sd)
    z = torch.randn(16, 3, 4, 6, generator=torch.Generator().manual_seed(VAE_SEED))
    scale = ov.latent_scale()
    with torch.no_grad():
        full = m.decode(z.unsqueeze(0), scale).float().clamp(-1, 1)[0]
        a = m.decode_chunk(z[:, :2].unsqueeze(0), scale, True).float().clamp(-1, 1)[0]
        b = m.decode_chunk(z[:, 2:].unsqueeze(0), scale, False).float().clamp(-1, 1)[0]
    return dict(cfg=VAE_CFG, seed=VAE_SEED, z=z, out=full, out_chunks=torch.cat([a, b], dim=1),
                checksum=sum(float(v.abs().sum()) for v in params.values()))


ROPE_BF16 = dict(grid=(3, 5, 7), start_frame=9, heads=2, seed=8)


def run_rope_bf16(mf):
    """The reference's RoPE rotation in its bf16 mode (mark_bf16_rope, model_fast.py:1000-1003: what every forward
    of a 4,096-token or larger chunk switches on) on seeded bf16 q rows: grids built in bf16 (:878-931) and
    causal_rope_apply_rotation (:933-979) with ROPE_DTYPE bf16."""
    f, h, w = ROPE_BF16["grid"]
    L, H, d = f * h * w, ROPE_BF16["heads"], 128
    g = torch.Generator().manual_seed(ROPE_BF16["seed"])
    x = torch.randn(L, H, d, generator=g).to(torch.bfloat16)
    freqs = torch.cat([mf.rope_params(1024, d - 4 * (d // 6)), mf.rope_params(1024, 2 * (d // 6)),
                       mf.rope_params(1024, 2 * (d // 6))], dim=1)
    cos_g, sin_g = mf._causal_rope_grids_build(freqs, torch.tensor([[f, h, w]]), "cpu", ROPE_BF16["start_frame"],
                                               dtype=torch.bfloat16)
    saved = mf.ROPE_DTYPE
    mf.mark_bf16_rope()
    try:
        out = mf.causal_rope_apply_rotation(x.unsqueeze(0), [(f, h, w)], cos_g, sin_g)[0]
    finally:
        mf.ROPE_DTYPE = saved
    return dict(case=ROPE_BF16, x=x, out=out.clone())


def main():
    if not REF or not os.path.isdir(os.path.join(REF, "wan")):
        raise SystemExit("set LBW_REFERENCE to the reference checkout (the directory holding wan/)")
    install_shims()
    with contextlib.redirect_stdout(sys.stderr):
        import wan.modules.model_fast as mf
        import wan.modules.attention as attn_mod
        import wan.modules.chunked_kv_cache as ckv
    if sys.argv[1:] == ["rope_bf16"]:       # only this fixture
        torch.save(run_rope_bf16(mf), os.path.join(HERE, "rope_bf16.pt"))
        print("rope_bf16 saved")
        return
    torch.manual_seed(0)
    for name, case in CASES.items():
        res = run_block(mf, case)
        torch.save(res, os.path.join(HERE, f"{name}.pt"))
        print(name, "x", tuple(res["x"].shape), "saved")
    res = run_dedup(attn_mod, mf)
    torch.save(res, os.path.join(HERE, "cross_dedup.pt"))
    print("cross_dedup saved")
    torch.save(run_cam(mf), os.path.join(HERE, "cam_film.pt"))
    print("cam_film saved")
    torch.save(run_model(mf, ckv), os.path.join(HERE, "model_forward.pt"))
    print("model_forward saved")
    table = {(i, n): ckv.chunk_routing(i, n) for n in (1, 2, 3, 4, 7) for i in range(0, 12)}
    torch.save(table, os.path.join(HERE, "chunk_routing.pt"))
    print("chunk_routing saved")
    torch.save(run_vae(), os.path.join(HERE, "vae_decode.pt"))
    print("vae_decode saved")
    torch.save(run_rope_bf16(mf), os.path.join(HERE, "rope_bf16.pt"))
    print("rope_bf16 saved")


if __name__ == "__main__":
    main()
