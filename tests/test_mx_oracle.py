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


def test_e5m2_scale_and_roundtrip():
    x = torch.zeros(3, 32)
    x[0, 0] = 57344.0        # 1.75 * 2^15 -> s = 0
    x[1, 4] = 1.0            # s = -15
    _, s = mx.quantize(x, "e5m2")
    assert s[:, 0].tolist() == [0, -15, -127]
    codes = torch.arange(256, dtype=torch.uint8).view(torch.float8_e5m2).float()
    codes = codes[torch.isfinite(codes)][:224].reshape(7, 32)
    codes[:, 0] = 57344.0    # pin each block's scale to 2^0
    assert torch.equal(mx.qdq(codes, "e5m2"), codes)
    y = torch.zeros(1, 32)
    # saturation; ties between neighbours 8192 apart go to the even mantissa: 45056 -> 49152 (mantissa 10),
    # 36864 -> 32768 (mantissa 00)
    y[0, 0], y[0, 1], y[0, 2] = 60000.0, 45056.0, 36864.0
    q = mx.qdq(y, "e5m2")
    assert q[0, :3].tolist() == [57344.0, 49152.0, 32768.0]


def test_e2m1_grid_ties_and_saturation():
    v = torch.tensor([0.2, 0.25, 0.3, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.5, 7.0, 100.0, -0.75, -5.0])
    want = torch.tensor([0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, 6.0, -1.0, -4.0])
    assert torch.equal(mx.e2m1_round(v), want)
    grid = torch.tensor(mx.E2M1_GRID)
    assert torch.equal(mx.e2m1_round(grid), grid) and torch.equal(mx.e2m1_round(-grid), -grid)


def test_e2m1_scale_codes_and_packing():
    x = torch.zeros(2, 32)
    x[0, 0] = 6.0            # 1.5 * 2^2 -> s = 0
    x[1, 0] = 1.0            # s = -2
    q, s = mx.quantize(x, "e2m1")
    assert s[:, 0].tolist() == [0, -2]
    vals = torch.tensor([0.5, -1.5, 3.0, -6.0] * 8)
    codes = mx.e2m1_codes(vals)
    assert codes[:4].tolist() == [0b0001, 0b1011, 0b0101, 0b1111]
    packed = mx.e2m1_pack(codes)
    assert packed[:2].tolist() == [0b1011_0001, 0b1111_0101]
    assert torch.equal(mx.e2m1_unpack(packed), vals)
    g = torch.Generator().manual_seed(1)
    w = torch.randn(64, 256, generator=g)
    qd = mx.qdq(w, "e2m1")
    assert (qd - w).norm() / w.norm() < 0.2          # 4-bit elements
    q, s = mx.quantize(w, "e2m1")
    assert torch.equal(mx.e2m1_unpack(mx.e2m1_pack(mx.e2m1_codes(q))).abs(), q.abs())
