"""ctypes binding of liblbw.so (the C ABI declared in include/lbw.h).

The library is the product path: if it is missing or fails to load, every op raises; there is no
CPU or PyTorch fallback. Status codes map to exceptions the way the reference's wrappers report
errors (wan/modules/attention.py:86-90, :209-210, :255-262): ValueError for bad arguments or
shapes, RuntimeError for device/runtime failures.
"""
import ctypes
import os
import re

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblbw.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "lbw.h")

LBW_OK, LBW_ERR_INVALID, LBW_ERR_SHAPE, LBW_ERR_ALIGN, LBW_ERR_CUDA, LBW_ERR_TIMEOUT, LBW_ERR_UNSUPPORTED = range(7)

_vp, _i, _ll, _f, _fp = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.POINTER(ctypes.c_float)

SIGNATURES = {
    "lbw_version": ([], _i),
    "lbw_last_error": ([ctypes.c_char_p, ctypes.c_size_t], _i),
    "lbw_status_string": ([_i], ctypes.c_char_p),
    "lbw_check_device_status": ([_vp, ctypes.POINTER(_i)], _i),
    "lbw_init": ([_i], _i),
    "lbw_destroy": ([_i], _i),
    "lbw_chunk_attention": ([_vp, _ll, _i, _i, _vp, _vp, _vp, _i, _ll, _vp, _f, _vp, _ll, _vp], _i),
    "lbw_gemm_bf16": ([_vp, _ll, _vp, _ll, _vp, _vp, _ll, _i, _i, _i, _vp], _i),
    "lbw_qkv_proj": ([_vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _ll, _i, _vp], _i),
    "lbw_linear_rowss": ([_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_linear_residual": ([_vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp], _i),
    "lbw_linear_gelu": ([_vp, _vp, _vp, _i, _i, _i, _vp, _i, _vp], _i),
    "lbw_layernorm_mod": ([_vp, _i, _i, _f, _vp, _vp, _vp, _vp, _i, _vp, _vp], _i),
    "lbw_rmsnorm_rope": ([_vp, _vp, _vp, _i, _i, _f, _vp, _vp, _i, _i, _i, _i, _vp, _ll, _i, _vp], _i),
    "lbw_qk_rmsnorm_rope": ([_vp, _vp, _vp, _vp, _ll, _i, _vp, _vp, _vp, _vp, _ll, _i, _i, _i, _f, _vp, _vp, _i, _i,
                             _i, _i, _vp], _i),
    "lbw_rmsnorm_rope_dt": ([_vp, _vp, _vp, _i, _i, _f, _vp, _vp, _i, _i, _i, _i, _vp, _ll, _i, _i, _vp], _i),
    "lbw_qk_rmsnorm_rope_dt": ([_vp, _vp, _vp, _vp, _ll, _i, _vp, _vp, _vp, _vp, _ll, _i, _i, _i, _f, _vp, _vp, _i, _i,
                                _i, _i, _i, _vp], _i),
    "lbw_mx_quantize": ([_vp, _i, _i, _vp, _vp, _vp, _vp], _i),
    "lbw_mx_quantize_fmt": ([_vp, _i, _i, _i, _vp, _vp, _vp, _vp], _i),
    "lbw_mx_linear_fmt": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_linear_rmsnorm_noalloc": ([_vp, _vp, _vp, _vp, _i, _i, _i, _f, _vp, _vp], _i),
    "lbw_chunk_attention_partial": ([_vp, _ll, _i, _i, _vp, _vp, _vp, _i, _ll, _vp, _f, _i, _vp, _vp, _i, _vp], _i),
    "lbw_attention_merge": ([_vp, _vp, _i, _i, _i, _vp, _ll, _vp], _i),
    "lbw_attention_tail_plan": ([_i, _i, _vp, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)], _i),
    "lbw_chunk_attention_tail": ([_vp, _ll, _i, _i, _vp, _vp, _vp, _i, _ll, _vp, _f, _vp, _ll, _i, _vp, _vp, _ll,
                                  _vp, ctypes.c_uint, _i, _vp], _i),
    "lbw_linear_act": ([_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_layernorm_mod_mx": ([_vp, _i, _i, _f, _vp, _vp, _vp, _vp, _vp], _i),
    "lbw_mx_linear": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp], _i),
    "lbw_mx_linear_gelu": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_mx_linear_residual": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_layernorm_mod_mx_fmt": ([_vp, _i, _i, _f, _vp, _vp, _i, _vp, _vp, _vp], _i),
    "lbw_layernorm_affine_mx_fmt": ([_vp, _i, _i, _f, _vp, _vp, _i, _vp, _vp, _vp], _i),
    "lbw_mx_qkv_proj_fmt": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _ll, _i, _vp], _i),
    "lbw_mx_linear_rowss_fmt": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_mx_linear_residual_film_fmt": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp], _i),
    "lbw_mx_linear_act_fmt": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_mx_linear_gelu_fmt": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_mx_linear_residual_fmt": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_layernorm_affine_mx": ([_vp, _i, _i, _f, _vp, _vp, _vp, _vp, _vp], _i),
    "lbw_mx_qkv_proj": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _vp, _vp, _vp, _vp, _vp, _ll, _i, _vp], _i),
    "lbw_mx_linear_rowss": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_mx_linear_residual_film": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp], _i),
    "lbw_mx_linear_act": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_vae_conv": ([_vp, _ll, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp], _i),
    "lbw_vae_conv_rms": ([_vp, _ll, _i, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp], _i),
    "lbw_vae_rms_silu": ([_vp, _ll, _i, _i, _vp, _i, _vp, _vp], _i),
    "lbw_vae_upsample2x": ([_vp, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_vae_time_interleave": ([_vp, _i, _ll, _i, _vp, _vp], _i),
    "lbw_vae_gather": ([_vp, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_vae_scatter_add": ([_vp, _vp, _i, _i, _i, _i, _vp, _vp], _i),
    "lbw_gemm_f32": ([_vp, _ll, _vp, _ll, _vp, _ll, _i, _i, _i, _vp], _i),
    "lbw_softmax_rows": ([_vp, _ll, _i, _i, _i, _f, _vp, _ll, _vp], _i),
    "lbw_transpose_bf16": ([_vp, _ll, _i, _i, _vp, _ll, _vp], _i),
    "lbw_chunk_attention_gated": ([_vp, _ll, _i, _i, _vp, _vp, _vp, _i, _ll, _f, _vp, _ll, _i, _vp, _vp, _i, _vp,
                                   ctypes.c_uint, _i, _vp], _i),
    "lbw_peer_buffer_create": ([_ll, ctypes.POINTER(_vp), _vp], _i),
    "lbw_peer_buffer_open": ([_vp, ctypes.POINTER(_vp)], _i),
    "lbw_peer_buffer_close": ([_vp, _i], _i),
    "lbw_host_flags_register": ([_vp, _ll, ctypes.POINTER(_vp)], _i),
    "lbw_host_flags_unregister": ([_vp], _i),
    "lbw_sp_kv_stage": ([ctypes.POINTER(_vp), _vp, _i, _i, ctypes.c_uint, _vp, _vp, _ll, _i, _i, _vp], _i),
    "lbw_sp_kv_gather": ([ctypes.POINTER(_vp), _vp, _i, _i, ctypes.c_uint, _vp, _vp, _ll, _i, _i, _vp], _i),
}

_lib = None


class LbwError(RuntimeError):
    pass


def load():
    """Loads liblbw.so once; raises if it was not built (run __graft_entry__.build())."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise LbwError(f"{LIB_PATH} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    _lib = lib
    return lib


def header_symbols(path=HEADER):
    """Names of every function declared in include/lbw.h."""
    txt = open(path).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(lbw_\w+)\s*\(", txt, re.M)))


def last_error():
    buf = ctypes.create_string_buffer(1024)
    load().lbw_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


# Entry points called successfully (each enqueues one kernel of liblbw.so, except lbw_linear_rmsnorm_noalloc, which
# enqueues two, and lbw_chunk_attention_tail, which enqueues two when it cuts windows); bench.py reads this for its
# launch count.
CALLS = [0]


def check(rc, what, launches=1):
    """Raises on a non-zero status; on success counts `launches` kernels enqueued by the call."""
    if rc == LBW_OK:
        if what not in ("device status", "lbw_init", "lbw_destroy", "attention_tail_plan"):
            CALLS[0] += launches
        return
    msg = f"{what}: {last_error()} (status {rc})"
    if rc in (LBW_ERR_INVALID, LBW_ERR_SHAPE, LBW_ERR_ALIGN, LBW_ERR_UNSUPPORTED):
        raise ValueError(msg)
    raise LbwError(msg)


def ptr(t):
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream_of(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def check_device_status(stream=None):
    """Synchronises the stream and raises LbwError if a kernel's bounded wait ran out."""
    code = ctypes.c_int(0)
    check(load().lbw_check_device_status(stream if stream is not None else stream_of(), ctypes.byref(code)),
          "device status")
    return code.value


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("lbw ops take CUDA tensors only (there is no CPU path)")


def init_device(device=None):
    """lbw_init: makes the library's per-device state (status word, peer pull streams) on `device` now."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    check(load().lbw_init(dev.index if dev.index is not None else torch.cuda.current_device()), "lbw_init")


def destroy_device(device=None):
    """lbw_destroy: waits for `device`, then releases the library's per-device state there."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    check(load().lbw_destroy(dev.index if dev.index is not None else torch.cuda.current_device()), "lbw_destroy")
