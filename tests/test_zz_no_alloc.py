"""The allocation-free entry point lbw_linear_rmsnorm_noalloc, called through the C ABI.

It serves callers that may not allocate device memory (runtimes that own all of HBM through their
own pool, plugins hosted by a framework without an allocator for them): its row-sum scratch and its
status word are fixed arrays inside liblbw.so. Its output must match the allocating pair
lbw_linear_rowss + lbw_rmsnorm_rope (no RoPE) and the CPU oracle's nn.Linear + WanRMSNorm on consecutive
calls, which also shows that each call clears the rows of the shared array it uses. Kept in its own
file, collected last.
"""
import ctypes

import pytest
import torch

from conftest import rel_l2
from oracle import block as ob

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _noalloc(lib, a, w, b, gamma, eps, out):
    import lbw_b200._lib as L
    m, k = a.shape
    n = w.shape[0]
    return lib.lbw_linear_rmsnorm_noalloc(L.ptr(a), L.ptr(w), L.ptr(b), L.ptr(gamma), m, n, k, ctypes.c_float(eps),
                                          L.ptr(out), L.stream_of(a.device))


def test_noalloc_matches_allocating_path_and_oracle_twice(cuda_dev):
    import lbw_b200._lib as L
    import lbw_b200.kernels as K
    lib = L.load()
    eps = 1e-6
    g = torch.Generator().manual_seed(31)
    for m, n, k in ((333, 512, 256), (1200, 384, 512)):   # two calls in a row, different rows
        a = torch.randn(m, k, generator=g).to(BF)
        w = (torch.randn(n, k, generator=g) * 0.05).to(BF)
        b = (torch.randn(n, generator=g) * 0.05).to(BF)
        gamma = (1 + 0.02 * torch.randn(n, generator=g)).to(BF)
        ad, wd, bd, gd = (t.to(cuda_dev) for t in (a, w, b, gamma))
        out = torch.empty(m, n, dtype=BF, device=cuda_dev)
        L.check(_noalloc(lib, ad, wd, bd, gd, eps, out), "linear_rmsnorm_noalloc")
        code = L.check_device_status()          # no timeout recorded in either status word
        assert code == 0
        raw = torch.empty(m, n, dtype=BF, device=cuda_dev)
        ss = torch.empty(m, dtype=torch.float32, device=cuda_dev)
        ref = torch.empty(m, n, dtype=BF, device=cuda_dev)
        K.linear_rowss(ad, wd, bd, raw, ss)
        K.rmsnorm_rope(raw, ss, gd, eps, ref)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert rel_l2(out, ref) < 2e-3
        oracle = ob.rms_norm(ob.linear(a, w, b), gamma, eps)    # nn.Linear then WanRMSNorm, on the CPU
        assert rel_l2(out, oracle) < 1e-2


def test_noalloc_rejects_rows_beyond_its_scratch(cuda_dev):
    import lbw_b200._lib as L
    lib = L.load()
    rc = lib.lbw_linear_rmsnorm_noalloc(ctypes.c_void_p(256), ctypes.c_void_p(256), None, ctypes.c_void_p(256),
                                        65537, 256, 256, ctypes.c_float(1e-6), ctypes.c_void_p(256), None)
    assert rc == L.LBW_ERR_SHAPE
    assert "at most 65536 rows" in L.last_error()
