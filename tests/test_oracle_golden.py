"""Pins the CPU oracle (oracle/) to fixtures produced by the reference's own code
(tests/golden/make_golden.py running wan/modules/model_fast.py CausalWanAttentionBlock on CPU)."""
import pytest
import torch

from conftest import load_golden, max_abs, rel_l2
from oracle import block as ob
from oracle.inputs import BlockCase, make_case
from tests.golden.make_golden import checksum


@pytest.mark.parametrize("name", ["block_flat", "block_peaked", "block_nofilm"])
def test_block_matches_reference(name):
    g = load_golden(name)
    case = BlockCase(**g["case"])
    p, inp = make_case(case)
    assert abs(checksum(p, inp) - g["checksum"]) <= 1e-4 * g["checksum"], "input generator drifted"
    cos, sin = ob.rope_grid(ob.rope_freqs(), case.grid, case.start_frame)
    assert torch.equal(cos, g["rope_cos"]) and torch.equal(sin, g["rope_sin"])
    ck, cv = ob.cross_kv(p, inp["context"])
    assert rel_l2(ck, g["ctx_k"]) < 1e-3 and rel_l2(cv, g["ctx_v"]) < 1e-3
    r = ob.block_forward(p, inp["x"], inp["e0"], inp["k_lead"], inp["v_lead"], ck, cv, cos, sin, film=inp["film"],
                         return_all=True)
    assert rel_l2(r["x"], g["x"]) < 1e-3
    assert rel_l2(r["x"] - inp["x"], g["x"] - inp["x"]) < 1e-2
    assert max_abs(r["x"], g["x"]) < 5e-3
    assert rel_l2(r["k"], g["k_dest"]) < 1e-3 and rel_l2(r["v"], g["v_dest"]) < 1e-3


def test_rope_bf16_matches_reference():
    """The rotation in the reference's bf16 RoPE mode (what every forward of a chunk of 4,096 or more tokens switches
    on): bf16 grids and bf16 products and sums, bit-identical to causal_rope_apply_rotation with ROPE_DTYPE bf16;
    the fp32 rotation of the same rows differs."""
    g = load_golden("rope_bf16")
    f, h, w = g["case"]["grid"]
    cos, sin = ob.rope_grid(ob.rope_freqs(), (f, h, w), g["case"]["start_frame"])
    got = ob.rope_apply(g["x"], cos, sin, torch.bfloat16)
    assert got.dtype == torch.bfloat16 and torch.equal(got, g["out"])
    assert not torch.equal(ob.rope_apply(g["x"], cos, sin), g["out"])


def test_rope_dtype_switch_follows_the_reference():
    """lbw_b200.rope.ROPE_DTYPE: fp32 until a forward sees seq_len >= 4096, then bf16 for the rest of the process
    (model_fast.py:1144-1148, :1000-1003)."""
    import lbw_b200.rope as R
    saved = R.ROPE_DTYPE
    try:
        R.ROPE_DTYPE = torch.float32
        R.set_bf16_rope_for_forward(4095)
        assert R.ROPE_DTYPE == torch.float32
        R.set_bf16_rope_for_forward(4096)
        assert R.ROPE_DTYPE == torch.bfloat16
        R.set_bf16_rope_for_forward(100)
        assert R.ROPE_DTYPE == torch.bfloat16
    finally:
        R.ROPE_DTYPE = saved


def test_cross_dedup_matches_reference():
    g = load_golden("cross_dedup")
    bias = ob.cross_dedup_bias(g["ctx_k"], g["ctx_v"], g["kc"])
    assert torch.allclose(bias, g["bias"])
    out = ob.attention(g["q"], g["ctx_k"][:g["kc"]], g["ctx_v"][:g["kc"]], key_bias=bias)
    assert rel_l2(out, g["out"]) < 5e-3
    # dedup with the log-multiplicity bias equals attention over the full duplicated context
    assert rel_l2(out, g["full"]) < 1e-2


def test_chunk_routing_table():
    import lbw_b200.chunked_kv_cache as ckv
    table = load_golden("chunk_routing")
    for (i, n), want in table.items():
        assert ckv.chunk_routing(i, n) == want, (i, n)


def test_cam_film_matches_reference():
    g = load_golden("cam_film")
    case = BlockCase(**g["case"])
    p, inp = make_case(case)
    assert abs(checksum(p, inp) - g["checksum"]) <= 1e-4 * g["checksum"]
    scale, shift = ob.cam_film(p, inp["cam"])
    assert rel_l2(scale, g["scale"]) < 2e-3 and rel_l2(shift, g["shift"]) < 2e-3


def test_model_forward_matches_reference():
    """The oracle's whole WanModelFast.forward (embeddings, camera FiLM, 2 blocks on the chunked cache, head,
    unpatchify) against the reference's own forward on the same seeded inputs."""
    from oracle import model as om
    from oracle.inputs import ModelCase, make_model_case
    import lbw_b200.chunked_kv_cache as routing
    g = load_golden("model_forward")
    case = ModelCase(**g["case"])
    sd, inp = make_model_case(case)
    out, k_dest, v_dest, ctx_k, ctx_v = om.model_forward(sd, inp, case, routing.chunk_routing)
    assert (g["dest"], g["leading"]) == routing.chunk_routing(case.chunk_index, case.n_chunks)
    assert rel_l2(out, g["out"]) < 2e-3 and max_abs(out, g["out"]) < 2e-2
    for i in range(case.layers):
        assert rel_l2(k_dest[i], g["k_dest"][i]) < 1e-2 and rel_l2(v_dest[i], g["v_dest"][i]) < 1e-2
        assert rel_l2(ctx_k[i], g["ctx_k"][i]) < 1e-2 and rel_l2(ctx_v[i], g["ctx_v"][i]) < 1e-2
    # a forward called with seq_len >= 4096 rotates in bf16, as the reference's: the roped K differs, V does not
    _, kb, vb, _, _ = om.model_forward(sd, inp, case, routing.chunk_routing, seq_len=4096)
    _, kb2, _, _, _ = om.model_forward(sd, inp, case, routing.chunk_routing, rope_dtype=torch.bfloat16)
    assert torch.equal(kb[0], kb2[0]) and not torch.equal(kb[0], k_dest[0]) and torch.equal(vb[0], v_dest[0])


def test_oracle_vae_decode_vs_reference_golden():
    """oracle.vae (the Wan 2.1 decoder restated) against the reference's WanVAE_.decode and a two-call
    decode_chunk of the same latent (tests/golden/vae_decode.pt)."""
    from oracle import vae as ov
    g = load_golden("vae_decode")
    p = ov.make_params(g["seed"], **g["cfg"])
    assert abs(sum(float(v.abs().sum()) for v in p.values()) - g["checksum"]) < 1e-3 * g["checksum"]
    out, _ = ov.decode(p, g["z"], **g["cfg"])
    assert out.shape == g["out"].shape == (3, 9, 32, 48)
    assert rel_l2(out, g["out"]) < 1e-5
    a, dec = ov.decode(p, g["z"][:, :2], **g["cfg"])
    b, _ = ov.decode(p, g["z"][:, 2:], decoder=dec, **g["cfg"])
    assert rel_l2(torch.cat([a, b], dim=1), g["out_chunks"]) < 1e-5
