"""Host side of the MX element formats: the format table of include/lbw.h and the Python wrappers agree, and the
emulation's E2M1 packing round-trips (no GPU needed)."""
import re

import torch

from oracle import mx as omx


def test_format_enum_matches_header():
    import os
    import lbw_b200.kernels as K
    hdr = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "lbw.h")).read()
    enum = dict((name.lower(), int(v)) for name, v in re.findall(r"LBW_MX_(E\dM\d)\s*=\s*(\d)", hdr))
    assert enum == K.MX_FORMATS


def test_row_bytes():
    import lbw_b200.kernels as K
    assert K.mx_row_bytes(512, "e4m3") == 512 and K.mx_row_bytes(512, "e5m2") == 512
    assert K.mx_row_bytes(512, "e2m1") == 256


def test_e2m1_pack_round_trip():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 64, generator=g) * 3
    q, s = omx.quantize(x, "e2m1")
    packed = omx.e2m1_pack(omx.e2m1_codes(q))
    assert packed.shape == (4, 32) and packed.dtype == torch.uint8
    assert torch.equal(omx.e2m1_unpack(packed), q)


def test_ffn_mx_reads_lingbot_mx_fp8():
    """ffn_mx takes its element format from LINGBOT_MX_FP8 at import, as the reference's kernels/ffn_mx.py:8,18
    does, and rejects a value the reference does not accept."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = ("import __graft_entry__; __graft_entry__.load_package(); import lbw_b200.ffn_mx as FM; print(FM.FMT)")
    for val, want in (("float8_e5m2", "e5m2"), ("float8_e4m3fn", "e4m3"), (None, "e4m3")):
        env = dict(os.environ)
        env.pop("LINGBOT_MX_FP8", None)
        if val:
            env["LINGBOT_MX_FP8"] = val
        out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True)
        assert out.returncode == 0 and out.stdout.strip() == want, out.stderr
    env = dict(os.environ, LINGBOT_MX_FP8="float16")
    out = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True)
    assert out.returncode != 0 and "LINGBOT_MX_FP8" in out.stderr
