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
