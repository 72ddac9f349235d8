"""OCP MX v1.0 E4M3 emulation (oracle/mx.py): spec properties."""
import torch

from oracle import mx


def test_scale_is_floor_log2_minus_8():
    x = torch.zeros(4, 32)
    x[0, 3] = 448.0          # 2^8 * 1.75 -> s = 0
    x[1, 0] = 1.0            # s = -8
    x[2, 5] = -3.0e-3        # floor(log2) = -9 -> s = -17
    _, s = mx.quantize(x)
    assert s[:, 0].tolist() == [0, -8, -17, -127]


def test_roundtrip_exact_for_representable_values():
    codes = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float()
    codes = codes[torch.isfinite(codes)][:224].reshape(7, 32)
    codes[:, 0] = 448.0      # pin each block's scale to 2^0
    assert torch.equal(mx.qdq(codes), codes)


def test_saturation_and_rne():
    x = torch.zeros(1, 32)
    x[0, 0] = 500.0          # amax 500 -> s = 0; 500 saturates to 448
    x[0, 1] = 17.0           # between 16 and 18 (E4M3 step 2 there): ties to even -> 16
    x[0, 2] = 19.0           # tie 18/20 -> 20
    y = mx.qdq(x)
    assert y[0, 0] == 448.0 and y[0, 1] == 16.0 and y[0, 2] == 20.0


def test_zero_block_and_tiled_scales():
    x = torch.randn(130, 256)
    x[1] = 0
    q, s = mx.quantize(x)
    assert (s[1] == -127).all() and (q[1].float() == 0).all()
    t = mx.scales_tiled(s, 256)
    assert t.numel() == 256 * 8
    assert int(t[mx.sf_offset(129, 7, 256)]) == int(s[129, 7]) + 127
    assert int(t[mx.sf_offset(131, 0, 256)]) == 0      # padded row
