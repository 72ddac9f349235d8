"""Host-side logic and the C ABI library (no GPU needed)."""
import ctypes

import pytest
import torch

import lbw_b200._lib as L
import lbw_b200.chunked_kv_cache as ckv
import lbw_b200.rope as rope
import lbw_b200.sp as sp
from oracle import block as ob


@pytest.fixture(scope="module")
def lib():
    import __graft_entry__
    __graft_entry__.build()
    return L.load()


def test_library_exports_every_header_symbol(lib):
    names = L.header_symbols()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert lib.lbw_version() == 1
    assert lib.lbw_status_string(5) == b"device wait timed out"


def test_argument_errors_are_reported_without_gpu(lib):
    # shape checks run before any CUDA call
    rc = lib.lbw_gemm_bf16(None, 64, None, 64, None, ctypes.c_void_p(16), 64, 128, 256, 100, None)
    assert rc == L.LBW_ERR_SHAPE and "multiple of 64" in L.last_error()
    with pytest.raises(ValueError):
        L.check(rc, "gemm")
    rc = lib.lbw_chunk_attention(ctypes.c_void_p(16), 256, 10, 2, None, None, None, 0, 256, None, ctypes.c_float(1.0),
                                 ctypes.c_void_p(16), 256, None)
    assert rc == L.LBW_ERR_INVALID


def test_ops_refuse_cpu_tensors():
    import lbw_b200.kernels as K
    q = torch.zeros(128, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        K.chunk_attention(q, [q], [q])


def test_chunk_routing_published_table():
    # window 12 / chunk 3 -> 4 chunks (reference chunked_kv_cache.py:55-63)
    want = [(0, ()), (1, (0,)), (2, (0, 1)), (3, (0, 1, 2)), (1, (0, 2, 3)), (2, (0, 1, 3))]
    assert [ckv.chunk_routing(i, 4) for i in range(6)] == want
    assert ckv.num_chunks(12, 3) == 4 and ckv.num_chunks(-1, 3) == 0


def test_allocate_and_order():
    cache = ckv.allocate_self_kv_chunks(2, 1, 16, 2, 128, 3, torch.bfloat16, "cpu")
    ks, vs = ckv.ordered_chunks_by_block(cache, 2, (0, 1))
    assert len(ks) == 2 and ks[0][-1] is cache[0]["k"][2]
    assert ckv.chunk_bytes(cache) == 2 * 2 * 3 * 16 * 2 * 128 * 2
    with pytest.raises(ValueError):
        ckv.allocate_self_kv_chunks(1, 1, 16, 2, 128, 3, torch.bfloat16, "cpu", n_major=True)


@pytest.mark.parametrize("grid,start", [((3, 4, 6), 6), ((3, 30, 52), 18), ((1, 45, 80), 0)])
def test_rope_tables_match_reference_grid(grid, start):
    freqs = rope.rope_freqs()
    assert torch.equal(freqs[:1024], ob.rope_freqs())
    cos, sin = rope.rope_tables(freqs, grid, start, "cpu")
    gc, gs = ob.rope_grid(ob.rope_freqs(), grid, start)
    f, h, w = grid
    t = torch.arange(f * h * w)
    fi, hi, wi = t // (h * w), (t // w) % h, t % w
    p = torch.arange(64)
    idx = torch.where(p < 22, fi[:, None] * 22 + p, torch.where(p < 43, f * 22 + hi[:, None] * 21 + (p - 22),
                                                                  f * 22 + h * 21 + wi[:, None] * 21 + (p - 43)))
    assert torch.equal(cos[idx], gc) and torch.equal(sin[idx], gs)


def test_shard_range():
    assert sp.shard_range(10800, 3, 8) == (4050, 5400)
    with pytest.raises(ValueError):
        sp.shard_range(10, 0, 3)


def test_model_state_dict_keys_match_the_reference():
    """CausalWanModel carries exactly the reference WanModelFast parameter names (checked against the keys the
    golden generator loaded into the reference model), so a reference checkpoint loads unchanged."""
    import lbw_b200.model as M
    from oracle.inputs import ModelCase, make_model_case
    case = ModelCase()
    sd, _ = make_model_case(case)
    m = M.CausalWanModel(model_type="i2v", in_dim=case.in_dim, dim=case.dim, ffn_dim=case.ffn, freq_dim=case.freq_dim,
                         text_dim=case.text_dim, out_dim=case.out_dim, num_heads=case.heads, num_layers=case.layers,
                         text_len=case.text_len)
    assert set(m.state_dict()) == set(sd)
    for k, v in m.state_dict().items():
        assert tuple(v.shape) == tuple(sd[k].shape), k


def _write_checkpoint(tmp_path, sharded):
    import json
    from safetensors.torch import save_file
    from oracle.inputs import ModelCase, make_model_case
    case = ModelCase()
    sd, _ = make_model_case(case)
    d = tmp_path / "transformers"
    d.mkdir()
    cfg = dict(model_type="i2v", patch_size=[1, 2, 2], text_len=case.text_len, in_dim=case.in_dim, dim=case.dim,
               ffn_dim=case.ffn, freq_dim=case.freq_dim, text_dim=case.text_dim, out_dim=case.out_dim,
               num_heads=case.heads, num_layers=case.layers, qk_norm=True, cross_attn_norm=True, eps=1e-6)
    (d / "config.json").write_text(json.dumps(cfg))
    tensors = {k: v.contiguous() for k, v in sd.items()}
    if sharded:
        keys = sorted(tensors)
        halves = [keys[: len(keys) // 2], keys[len(keys) // 2:]]
        wmap = {}
        for i, ks in enumerate(halves):
            name = f"diffusion_pytorch_model-0000{i + 1}-of-00002.safetensors"
            save_file({k: tensors[k] for k in ks}, str(d / name))
            wmap.update({k: name for k in ks})
        (d / "diffusion_pytorch_model.safetensors.index.json").write_text(json.dumps({"weight_map": wmap}))
    else:
        save_file(tensors, str(d / "model.safetensors"))
    return case, sd


@pytest.mark.parametrize("sharded", [False, True])
def test_checkpoint_loader_reads_reference_layout(tmp_path, sharded):
    """A DiT folder laid out like the reference upload (transformers/, config.json, sharded safetensors + index)
    loads into CausalWanModel with every parameter, in the pipeline's dtypes, values unchanged."""
    import lbw_b200.checkpoint as ck
    case, sd = _write_checkpoint(tmp_path, sharded)
    model, unexpected = ck.load_model(str(tmp_path), device="cpu", pack=False)
    assert unexpected == []
    msd = model.state_dict()
    assert set(msd) == set(sd)
    for k, v in sd.items():
        assert torch.equal(msd[k].float(), v.float()), k
    assert msd["time_embedding.0.weight"].dtype == torch.float32 and msd["blocks.0.modulation"].dtype == torch.float32
    assert msd["blocks.1.self_attn.q.weight"].dtype == torch.bfloat16
    assert model.num_layers == case.layers and model.dim == case.dim


def test_checkpoint_loader_rejects_missing_and_misshapen(tmp_path):
    import lbw_b200.checkpoint as ck
    from safetensors.torch import load_file, save_file
    _write_checkpoint(tmp_path, sharded=False)
    path = tmp_path / "transformers" / "model.safetensors"
    t = load_file(str(path))
    t.pop("blocks.1.ffn.2.bias")
    save_file(t, str(path))
    with pytest.raises(ValueError, match="lacks 1 parameters"):
        ck.load_model(str(tmp_path), device="cpu", pack=False)
    t["blocks.1.ffn.2.bias"] = torch.zeros(7)
    save_file(t, str(path))
    with pytest.raises(ValueError, match="checkpoint shape"):
        ck.load_model(str(tmp_path), device="cpu", pack=False)


def test_lin_mx_options():
    """LINGBOT_LIN_MX / LINGBOT_LIN_MX_SKIP host logic: which Linears go to the MXFP8 GEMM."""
    import lbw_b200.block as B
    with torch.device("meta"):
        blk = B.CausalWanAttentionBlock(256, 512, 2, cross_attn_norm=True, ffn_mx=False, lin_mx=True,
                                        lin_mx_skip=("self_attn.o", "cam_scale_layer"))
        assert blk.ffn_mx                      # LIN_MX implies the MXFP8 FFN
        assert blk.mx_linears == frozenset(B.MX_LINEAR_NAMES) - {"self_attn.o", "cam_scale_layer"}
        assert B.CausalWanAttentionBlock(256, 512, 2).mx_linears == frozenset()
        with pytest.raises(ValueError, match="names no block Linear"):
            B.CausalWanAttentionBlock(256, 512, 2, lin_mx=True, lin_mx_skip=("ffn.0",))
        with pytest.raises(ValueError, match="all three or none"):
            B.CausalWanAttentionBlock(256, 512, 2, lin_mx=True, lin_mx_skip=("self_attn.k",))
        with pytest.raises(ValueError, match="mx_pipe"):
            B.CausalWanAttentionBlock(256, 512, 2, lin_mx=True, mx_pipe="bf16")


def test_oracle_lin_mx_changes_only_the_named_linears():
    """The oracle's LINGBOT_LIN_MX emulation: MXFP8 Linears move the block output by the MX quantisation error
    (a few percent of the update), and naming no Linear gives the MX-FFN block exactly."""
    from oracle.inputs import BlockCase, make_case
    import lbw_b200.block as B
    case = BlockCase(dim=256, ffn=512, grid=(2, 4, 6), n_lead=1, text_len=32, seed=41)
    p, inp = make_case(case)
    cos, sin = ob.rope_grid(ob.rope_freqs(), case.grid, case.start_frame)
    ck, cv = ob.cross_kv(p, inp["context"])
    args = (p, inp["x"], inp["e0"], inp["k_lead"], inp["v_lead"], ck, cv, cos, sin)
    base = ob.block_forward(*args, film=inp["film"], mx=True)
    assert torch.equal(ob.block_forward(*args, film=inp["film"], mx=True, mx_linears=()), base)
    ckm, cvm = ob.cross_kv(p, inp["context"], mx_linears=B.MX_LINEAR_NAMES)
    allmx = ob.block_forward(p, inp["x"], inp["e0"], inp["k_lead"], inp["v_lead"], ckm, cvm, cos, sin,
                             film=inp["film"], mx_linears=B.MX_LINEAR_NAMES)
    d = (allmx - base).norm() / (base - inp["x"]).norm()
    assert 1e-3 < d < 0.1


def test_vae_decoder_parameter_names_match_the_reference():
    """WanVAEDecoder carries conv2.* + decoder.* with the reference's names and shapes (the list in oracle.vae is
    checked against the reference's own WanVAE_ state dict when the golden is made), so a checkpoint loads as is."""
    import lbw_b200.vae as V
    from oracle import vae as ov
    for dim in (32, 96):
        m = V.WanVAEDecoder(dim=dim)
        got = {n: tuple(p.shape) for n, p in m.named_parameters()}
        assert got == {n: tuple(s) for n, s in ov.param_shapes(dim=dim)}
    with pytest.raises(ValueError, match="CUDA"):
        V.WanVAEDecoder(dim=32).prepare()


def test_vae_history_buffer_keeps_the_last_two_frames():
    """The per-layer causal buffer of the VAE decoder: after each call its frames 0-1 are the last two frames of
    the layer's whole input series (zeros before the first frame), whatever the number of frames per call."""
    import lbw_b200.vae as V
    P, c = 3, 2
    h = V._Hist(P, c, 4, "cpu")
    series = [torch.zeros(P, c, dtype=torch.bfloat16), torch.zeros(P, c, dtype=torch.bfloat16)]
    val = 1.0
    for t in (1, 1, 2, 4, 1, 4, 2):
        frames = [torch.full((P, c), val + i, dtype=torch.bfloat16) for i in range(t)]
        val += t
        h.slot(t).copy_(torch.cat(frames))
        assert torch.equal(h.buf[:2 * P], torch.cat(series[-2:]))      # what the convolution reads in front
        series += frames
        h.advance(t)
        assert torch.equal(h.buf[:2 * P], torch.cat(series[-2:]))


def _p(v=256):
    return ctypes.c_void_p(v)   # a 256-byte-aligned stand-in address: never dereferenced, the checks come first


@pytest.mark.parametrize("case", ["qk_null", "qk_width", "qk_grid", "rr_pair", "mx_fmt", "mx_k", "noalloc_rows",
                                  "noalloc_k", "vae_kernel", "vae_channels"])
def test_entry_points_validate_before_any_cuda_call(lib, case):
    """Each entry point rejects bad arguments with its status code and a message, before it touches CUDA (the
    reference's wrappers raise ValueError / RuntimeError the same way, wan/modules/attention.py:86-90)."""
    f, c, s = ctypes.c_float, ctypes.c_longlong, None
    calls = {
        "qk_null": (lambda: lib.lbw_qk_rmsnorm_rope(None, _p(), _p(), _p(), c(512), 0, _p(), _p(), _p(), _p(), c(512),
                                                     0, 4, 512, f(1e-6), None, None, 0, 0, 0, 0, s),
                    L.LBW_ERR_INVALID, "null"),
        "qk_width": (lambda: lib.lbw_qk_rmsnorm_rope(_p(), _p(), _p(), _p(), c(500), 0, _p(), _p(), _p(), _p(), c(500),
                                                      0, 4, 500, f(1e-6), None, None, 0, 0, 0, 0, s),
                     L.LBW_ERR_SHAPE, "multiple of 128"),
        "qk_grid": (lambda: lib.lbw_qk_rmsnorm_rope(_p(), _p(), _p(), _p(), c(512), 0, _p(), _p(), _p(), _p(), c(512), 0,
                                                     100, 512, f(1e-6), _p(), _p(), 3, 4, 6, 0, s),
                    L.LBW_ERR_SHAPE, "outside"),
        "rr_pair": (lambda: lib.lbw_rmsnorm_rope(_p(), _p(), _p(), 4, 512, f(1e-6), _p(), None, 1, 1, 1, 0, _p(),
                                                 c(512), 0, s),
                    L.LBW_ERR_INVALID, "cos/sin"),
        "mx_fmt": (lambda: lib.lbw_mx_quantize_fmt(_p(), 4, 128, 7, _p(), _p(), None, s), L.LBW_ERR_INVALID, "format"),
        "mx_k": (lambda: lib.lbw_mx_quantize_fmt(_p(), 4, 100, 0, _p(), _p(), None, s), L.LBW_ERR_SHAPE, "multiple"),
        "noalloc_rows": (lambda: lib.lbw_linear_rmsnorm_noalloc(_p(), _p(), None, _p(), 65537, 256, 256, f(1e-6),
                                                                _p(), s),
                         L.LBW_ERR_SHAPE, "at most 65536"),
        "noalloc_k": (lambda: lib.lbw_linear_rmsnorm_noalloc(_p(), _p(), None, _p(), 8, 256, 100, f(1e-6), _p(), s),
                      L.LBW_ERR_SHAPE, "K=100"),
        "vae_kernel": (lambda: lib.lbw_vae_conv(_p(), 1000, 64, _p(), None, 64, 2, 3, 3, 1, 4, 4, None, _p(), s),
                       L.LBW_ERR_SHAPE, "kernel"),
        "vae_channels": (lambda: lib.lbw_vae_conv(_p(), 1000, 60, _p(), None, 64, 3, 3, 3, 1, 4, 4, None, _p(), s),
                         L.LBW_ERR_SHAPE, "channels"),
    }
    fn, code, text = calls[case]
    assert fn() == code
    assert text in L.last_error()


def test_block_mx_format_options(monkeypatch):
    """mx_fp8 (LINGBOT_MX_FP8): E4M3 by default, E5M2 for the MX FFN and the LINGBOT_LIN_MX Linears; refused for the
    bf16-pipe variant (E4M3 only) and for a name the reference does not accept."""
    import lbw_b200.block as B
    mk = lambda **kw: B.CausalWanAttentionBlock(256, 512, 2, cross_attn_norm=True, **kw)  # noqa: E731
    assert mk().mx_fmt == "e4m3"
    assert mk(mx_fp8="float8_e5m2").mx_fmt == "e5m2"
    assert mk(mx_fp8="float8_e5m2", lin_mx=True).mx_fmt == "e5m2"
    with pytest.raises(ValueError, match="E4M3 only"):
        mk(mx_fp8="float8_e5m2", mx_pipe="bf16")
    with pytest.raises(ValueError, match="mx_fp8"):
        mk(mx_fp8="float16")
