"""Torch-tensor wrappers over the C ABI (one function per lbw_* entry point).

Every wrapper validates dtypes/devices, passes raw pointers and the current CUDA stream, and turns a
non-zero status into ValueError / LbwError. Outputs may be passed in (written in place) or are
allocated here.
"""
import ctypes
import math

import torch

from . import _lib
from ._lib import check, load, ptr, require_cuda, stream_of

BF16 = torch.bfloat16
HEAD_DIM = 128


def _tracing(eager):
    """True while torch.compile traces a graph (and the caller is not the operator's own implementation): the
    wrapper then calls the torch.ops.lbw operator (lbw_b200.ops) so that the kernel becomes a graph node."""
    return not eager and torch.compiler.is_compiling()


def _op(name):
    """torch.ops.lbw.<name> (registered when lbw_b200.ops is imported, as lbw_b200.block does)."""
    return getattr(torch.ops.lbw, name)


def _c(t, dtype=None):
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t


def _rows(t):
    """2-D [rows, cols] view of a [.., rows, heads, d] / [rows, cols] tensor (must be contiguous)."""
    _c(t)
    return t.reshape(-1, t.shape[-2] * t.shape[-1]) if t.dim() >= 3 else t


def chunk_attention(q, k_chunks, v_chunks, key_bias=None, out=None, softmax_scale=None, _eager=False):
    """q [Lq, H, 128] (or [1, Lq, H, 128] / [Lq, H*128]) bf16; chunks [L_i, H, 128]-like bf16 ->
    out [Lq, H*128] bf16 = softmax(q kᵀ * scale + bias) v over the concatenated chunks."""
    if _tracing(_eager):
        if out is None:
            out = torch.empty(q.numel() // (q.shape[-1] * (q.shape[-2] if q.dim() >= 3 else 1)),
                              q.shape[-1] * (q.shape[-2] if q.dim() >= 3 else 1), dtype=BF16, device=q.device)
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
        _op("chunk_attention")(q, list(k_chunks), list(v_chunks), key_bias, float(scale), out)
        return out
    require_cuda(q, *k_chunks, *v_chunks, key_bias, out)
    q2 = _rows(_c(q, BF16))
    lq, cols = q2.shape
    if cols % HEAD_DIM:
        raise ValueError("head_dim must be 128")
    heads = cols // HEAD_DIM
    n = len(k_chunks)
    if n != len(v_chunks) or n == 0:
        raise ValueError("need the same, non-zero number of K and V chunks")
    ks = [_rows(_c(k, BF16)) for k in k_chunks]
    vs = [_rows(_c(v, BF16)) for v in v_chunks]
    for k, v in zip(ks, vs):
        if k.shape != v.shape or k.shape[1] != cols:
            raise ValueError(f"chunk shape {tuple(k.shape)} / {tuple(v.shape)} does not match q width {cols}")
    if out is None:
        out = torch.empty(lq, cols, dtype=BF16, device=q.device)
    o2 = _rows(_c(out, BF16))
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for v in vs])
    rows = (ctypes.c_int * n)(*[k.shape[0] for k in ks])
    if key_bias is not None:
        key_bias = _c(key_bias, torch.float32)
        if key_bias.numel() != sum(k.shape[0] for k in ks):
            raise ValueError("key_bias needs one value per key")
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
    check(load().lbw_chunk_attention(ptr(q2), q2.stride(0), lq, heads, kp, vp, rows, n, cols, ptr(key_bias),
                                     ctypes.c_float(scale), ptr(o2), o2.stride(0), stream_of(q.device)),
          "chunk_attention")
    return out


def n_kv_tiles(chunk_rows):
    return sum((r + 127) // 128 for r in chunk_rows)


def attention_workspace(n_slots, q_rows, heads, device):
    """fp32 partial outputs [n_slots, q_rows, heads, 128] and (m, l) [n_slots, q_rows, heads, 2]."""
    return (torch.empty(n_slots, q_rows, heads, HEAD_DIM, dtype=torch.float32, device=device),
            torch.empty(n_slots, q_rows, heads, 2, dtype=torch.float32, device=device))


def chunk_attention_partial(q, k_chunks, v_chunks, n_splits, part_o, part_ml, slot0=0, key_bias=None,
                            softmax_scale=None, _eager=False):
    """Split-KV attention into workspace slots slot0 .. slot0 + n_splits - 1 (see lbw.h)."""
    if _tracing(_eager):
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
        _op("chunk_attention_partial")(q, list(k_chunks), list(v_chunks), int(n_splits), part_o, part_ml, int(slot0),
                                       key_bias, float(scale))
        return
    require_cuda(q, *k_chunks, *v_chunks, key_bias, part_o, part_ml)
    q2 = _rows(_c(q, BF16))
    lq, cols = q2.shape
    heads = cols // HEAD_DIM
    n = len(k_chunks)
    ks = [_rows(_c(k, BF16)) for k in k_chunks]
    vs = [_rows(_c(v, BF16)) for v in v_chunks]
    if part_o.shape[1:] != (lq, heads, HEAD_DIM) or part_ml.shape[1:] != (lq, heads, 2):
        raise ValueError("attention workspace does not match q")
    if slot0 < 0 or slot0 + n_splits > part_o.shape[0]:
        raise ValueError(f"slots {slot0}..{slot0 + n_splits - 1} outside a {part_o.shape[0]}-slot workspace")
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for v in vs])
    rows = (ctypes.c_int * n)(*[k.shape[0] for k in ks])
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
    check(load().lbw_chunk_attention_partial(ptr(q2), q2.stride(0), lq, heads, kp, vp, rows, n, cols, ptr(key_bias),
                                             ctypes.c_float(scale), int(n_splits), ptr(part_o), ptr(part_ml),
                                             int(slot0), stream_of(q.device)), "chunk_attention_partial")


def chunk_attention_gated(q, k_chunks, v_chunks, gate_flag_ptr, gate_value, gate_chunk, out=None, n_splits=1,
                          part_o=None, part_ml=None, slot0=0, softmax_scale=None):
    """chunk_attention (out) or chunk_attention_partial (part_o, part_ml) whose chunks gate_chunk.. are waited
    for in-kernel: loads from them start once the 32-bit word at gate_flag_ptr (a device address) has reached
    gate_value (see lbw.h)."""
    require_cuda(q, *k_chunks, *v_chunks, out, part_o, part_ml)
    q2 = _rows(_c(q, BF16))
    lq, cols = q2.shape
    heads = cols // HEAD_DIM
    n = len(k_chunks)
    ks = [_rows(_c(k, BF16)) for k in k_chunks]
    vs = [_rows(_c(v, BF16)) for v in v_chunks]
    o2 = None
    if out is not None:
        o2 = _rows(_c(out, BF16))
        if o2.shape[0] != lq or o2.shape[1] < cols:
            raise ValueError("chunk_attention_gated: out does not match q")
    else:
        if part_o is None or part_ml is None:
            raise ValueError("chunk_attention_gated: give out or the partial buffers")
        if part_o.shape[1:] != (lq, heads, HEAD_DIM) or part_ml.shape[1:] != (lq, heads, 2):
            raise ValueError("attention workspace does not match q")
        if slot0 < 0 or slot0 + n_splits > part_o.shape[0]:
            raise ValueError(f"slots {slot0}..{slot0 + n_splits - 1} outside a {part_o.shape[0]}-slot workspace")
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for v in vs])
    rows = (ctypes.c_int * n)(*[k.shape[0] for k in ks])
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
    check(load().lbw_chunk_attention_gated(ptr(q2), q2.stride(0), lq, heads, kp, vp, rows, n, cols,
                                           ctypes.c_float(scale), ptr(o2), o2.stride(0) if o2 is not None else 0,
                                           int(n_splits), ptr(part_o), ptr(part_ml), int(slot0),
                                           ctypes.c_void_p(gate_flag_ptr), ctypes.c_uint(gate_value), int(gate_chunk),
                                           stream_of(q.device)), "chunk_attention_gated")
    return out


_TAIL_PLANS = {}


def attention_tail_plan(q_rows, heads, chunk_rows, device, pieces=0):
    """(cut windows, pieces) of lbw_chunk_attention_tail on `device` (its SM count sets the waves); cached."""
    device = torch.device(device)
    key = (int(q_rows), int(heads), tuple(int(r) for r in chunk_rows), device.index, int(pieces))
    hit = _TAIL_PLANS.get(key)
    if hit is None:
        n = len(chunk_rows)
        rows = (ctypes.c_int * n)(*key[2])
        n_tail, used = ctypes.c_int(0), ctypes.c_int(0)
        with torch.cuda.device(device):
            check(load().lbw_attention_tail_plan(key[0], key[1], rows, n, key[4], ctypes.byref(n_tail),
                                                 ctypes.byref(used)), "attention_tail_plan")
        hit = _TAIL_PLANS[key] = (n_tail.value, used.value)
    return hit


def attention_tail_workspace(q_rows, heads, chunk_rows, device, pieces=0):
    """fp32 workspace (part_o [blocks, 256, 128], part_ml [blocks, 256, 2]) for chunk_attention_tail, or None
    when nothing is cut."""
    n_tail, used = attention_tail_plan(q_rows, heads, chunk_rows, device, pieces)
    if n_tail == 0:
        return None
    blocks = n_tail * used
    return (torch.empty(blocks, 256, HEAD_DIM, dtype=torch.float32, device=device),
            torch.empty(blocks, 256, 2, dtype=torch.float32, device=device))


def chunk_attention_tail(q, k_chunks, v_chunks, workspace, key_bias=None, out=None, pieces=0, gate_flag_ptr=None,
                         gate_value=0, gate_chunk=None, softmax_scale=None, _eager=False):
    """chunk_attention with the windows past the last full wave cut into key ranges (see lbw.h); `workspace`
    from attention_tail_workspace with the same pieces. With gate_flag_ptr, chunks gate_chunk.. are waited
    for in-kernel as in chunk_attention_gated."""
    if _tracing(_eager) and gate_flag_ptr is None:
        if out is None:
            raise ValueError("chunk_attention_tail: pass out= when compiling")
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
        part_o, part_ml = workspace if workspace is not None else (None, None)
        _op("chunk_attention_tail")(q, list(k_chunks), list(v_chunks), key_bias, float(scale), out, part_o, part_ml,
                                    int(pieces))
        return out
    require_cuda(q, *k_chunks, *v_chunks, key_bias, out)
    q2 = _rows(_c(q, BF16))
    lq, cols = q2.shape
    if cols % HEAD_DIM:
        raise ValueError("head_dim must be 128")
    heads = cols // HEAD_DIM
    n = len(k_chunks)
    if n != len(v_chunks) or n == 0:
        raise ValueError("need the same, non-zero number of K and V chunks")
    ks = [_rows(_c(k, BF16)) for k in k_chunks]
    vs = [_rows(_c(v, BF16)) for v in v_chunks]
    for k, v in zip(ks, vs):
        if k.shape != v.shape or k.shape[1] != cols:
            raise ValueError(f"chunk shape {tuple(k.shape)} / {tuple(v.shape)} does not match q width {cols}")
    if out is None:
        out = torch.empty(lq, cols, dtype=BF16, device=q.device)
    o2 = _rows(_c(out, BF16))
    if o2.shape[0] != lq or o2.shape[1] < cols:
        raise ValueError("chunk_attention_tail: out does not match q")
    part_o = part_ml = None
    blocks = 0
    if workspace is not None:
        part_o, part_ml = workspace
        require_cuda(part_o, part_ml)
        _c(part_o, torch.float32), _c(part_ml, torch.float32)
        if part_o.shape[1:] != (256, HEAD_DIM) or part_ml.shape[1:] != (256, 2) or part_o.shape[0] != part_ml.shape[0]:
            raise ValueError("chunk_attention_tail: workspace must be [blocks, 256, 128] and [blocks, 256, 2] fp32")
        blocks = part_o.shape[0]
    if key_bias is not None:
        key_bias = _c(key_bias, torch.float32)
        if key_bias.numel() != sum(k.shape[0] for k in ks):
            raise ValueError("key_bias needs one value per key")
    kp = (ctypes.c_void_p * n)(*[k.data_ptr() for k in ks])
    vp = (ctypes.c_void_p * n)(*[v.data_ptr() for v in vs])
    rows = (ctypes.c_int * n)(*[k.shape[0] for k in ks])
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(HEAD_DIM)
    gate_chunk = n if gate_flag_ptr is None else int(gate_chunk)
    n_tail, _ = attention_tail_plan(lq, heads, [k.shape[0] for k in ks], q.device, pieces)
    check(load().lbw_chunk_attention_tail(ptr(q2), q2.stride(0), lq, heads, kp, vp, rows, n, cols, ptr(key_bias),
                                          ctypes.c_float(scale), ptr(o2), o2.stride(0), int(pieces), ptr(part_o),
                                          ptr(part_ml), blocks, ctypes.c_void_p(gate_flag_ptr or 0),
                                          ctypes.c_uint(gate_value), gate_chunk, stream_of(q.device)),
          "chunk_attention_tail", launches=2 if n_tail else 1)
    return out


def attention_merge(part_o, part_ml, n_slots, out, _eager=False):
    if _tracing(_eager):
        _op("attention_merge")(part_o, part_ml, int(n_slots), out)
        return out
    require_cuda(part_o, part_ml, out)
    _, lq, heads, _ = part_o.shape
    o2 = _rows(_c(out, BF16))
    check(load().lbw_attention_merge(ptr(part_o), ptr(part_ml), int(n_slots), lq, heads, ptr(o2), o2.stride(0),
                                     stream_of(out.device)), "attention_merge")
    return out


def pick_kv_splits(q_rows, heads, n_tiles, sms=148, max_splits=4):
    """Fewest KV splits whose CTA count fills the last wave to >= 90% (else the best fill)."""
    blocks = (q_rows + 255) // 256 * heads
    best, best_eff = 1, 0.0
    for s in range(1, max_splits + 1):
        if s > n_tiles:
            break
        waves = blocks * s / sms
        eff = waves / math.ceil(waves)
        if eff >= 0.9:
            return s
        if eff > best_eff + 1e-9:
            best, best_eff = s, eff
    return best


def gemm_bf16(a, w, bias=None, out=None):
    require_cuda(a, w, bias, out)
    _c(a, BF16), _c(w, BF16)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError("gemm_bf16: K mismatch")
    if out is None:
        out = torch.empty(m, n, dtype=BF16, device=a.device)
    check(load().lbw_gemm_bf16(ptr(a), a.stride(0), ptr(w), w.stride(0), ptr(bias), ptr(out), out.stride(0), m, n,
                               k, stream_of(a.device)), "gemm_bf16")
    return out


def qkv_proj(h, w_qkv, b_qkv, q_raw, k_raw, ss_q, ss_k, v_out, v_row_off=0, _eager=False):
    if _tracing(_eager):
        _op("qkv_proj")(h, w_qkv, b_qkv, q_raw, k_raw, ss_q, ss_k, v_out, int(v_row_off))
        return
    require_cuda(h, w_qkv, b_qkv, q_raw, k_raw, ss_q, ss_k, v_out)
    m, c = h.shape
    v2 = _rows(v_out)
    if w_qkv.shape != (3 * c, c) or q_raw.shape != (m, c) or k_raw.shape != (m, c) or ss_q.numel() < m:
        raise ValueError("qkv_proj: shape mismatch")
    if v2.shape[1] != c or v_row_off < 0 or v_row_off + m > v2.shape[0]:
        raise ValueError(f"qkv_proj: rows {v_row_off}..{v_row_off + m} outside the V destination ({v2.shape[0]} rows)")
    check(load().lbw_qkv_proj(ptr(h), ptr(w_qkv), ptr(b_qkv), m, c, ptr(q_raw), ptr(k_raw), ptr(ss_q), ptr(ss_k),
                              ptr(v2), v2.stride(0), v_row_off, stream_of(h.device)), "qkv_proj")


def linear_rowss(a, w, bias, out, ss, _eager=False):
    if _tracing(_eager):
        _op("linear_rowss")(a, w, bias, out, ss)
        return out
    require_cuda(a, w, bias, out, ss)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or out.shape != (m, n) or ss.numel() < m:
        raise ValueError("linear_rowss: shape mismatch")
    check(load().lbw_linear_rowss(ptr(a), ptr(w), ptr(bias), m, n, k, ptr(out), ptr(ss), stream_of(a.device)),
          "linear_rowss")
    return out


def linear_residual(a, w, bias, x, gate=None, film_scale=None, film_shift=None, _eager=False):
    if _tracing(_eager):
        _op("linear_residual")(a, w, bias, x, gate, film_scale, film_shift)
        return x
    require_cuda(a, w, bias, x, gate, film_scale, film_shift)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or x.shape != (m, n) or x.dtype != torch.float32:
        raise ValueError("linear_residual: x must be fp32 [m, n]")
    for t in (film_scale, film_shift):
        if t is not None and (t.shape != (m, n) or t.dtype != BF16 or not t.is_contiguous()):
            raise ValueError("linear_residual: FiLM tensors must be contiguous bf16 [m, n]")
    check(load().lbw_linear_residual(ptr(a), ptr(w), ptr(bias), m, n, k, ptr(x), ptr(gate), ptr(film_scale),
                                     ptr(film_shift), stream_of(a.device)), "linear_residual")
    return x


def linear_act(a, w, bias=None, addend=None, silu=False, out=None):
    """bf16(act(bf16(a w^T + bias))) (+ addend): the camera-FiLM MLP layers."""
    require_cuda(a, w, bias, addend, out)
    _c(a, BF16), _c(w, BF16)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or (addend is not None and (addend.shape != (m, n) or addend.dtype != BF16)):
        raise ValueError("linear_act: shape mismatch")
    if addend is not None:
        _c(addend)
    if out is None:
        out = torch.empty(m, n, dtype=BF16, device=a.device)
    check(load().lbw_linear_act(ptr(a), ptr(w), ptr(bias), ptr(addend), int(bool(silu)), m, n, k, ptr(out),
                                stream_of(a.device)), "linear_act")
    return out


def linear_gelu(a, w, bias, out, mx_qdq, _eager=False):
    if _tracing(_eager):
        _op("linear_gelu")(a, w, bias, out, bool(mx_qdq))
        return out
    require_cuda(a, w, bias, out)
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or out.shape != (m, n):
        raise ValueError("linear_gelu: shape mismatch")
    check(load().lbw_linear_gelu(ptr(a), ptr(w), ptr(bias), m, n, k, ptr(out), int(mx_qdq), stream_of(a.device)),
          "linear_gelu")
    return out


def layernorm_mod(x, eps, out, scale=None, shift=None, weight=None, bias=None, mx_qdq=False, _eager=False):
    if _tracing(_eager):
        _op("layernorm_mod")(x, float(eps), out, scale, shift, weight, bias, bool(mx_qdq))
        return out
    require_cuda(x, out)
    _c(x, torch.float32)
    m, c = x.shape
    check(load().lbw_layernorm_mod(ptr(x), m, c, ctypes.c_float(eps), ptr(scale), ptr(shift), ptr(weight), ptr(bias),
                                   int(mx_qdq), ptr(out), stream_of(x.device)), "layernorm_mod")
    return out


def rmsnorm_rope(x, ss, gamma, eps, out, rope=None, grid=None, tok0=0, out_row_off=0, rope_bf16=False,
                 _eager=False):
    """rope = (cos, sin, n_frames) from rope.rope_tables; grid = (f, h, w). rope_bf16: the reference's bf16
    rotation (lbw.h LBW_ROPE_BF16; rope.ROPE_DTYPE), else fp32."""
    if _tracing(_eager):
        if rope is not None:
            _op("rmsnorm_rope")(x, ss, gamma, float(eps), out, rope[0], rope[1], int(rope[2]), int(grid[1]),
                                int(grid[2]), int(tok0), int(out_row_off), bool(rope_bf16))
        else:
            _op("rmsnorm_rope")(x, ss, gamma, float(eps), out, None, None, 0, 0, 0, int(tok0), int(out_row_off),
                                False)
        return out
    require_cuda(x, ss, gamma, out)
    m, c = x.shape
    o2 = _rows(out)
    if o2.shape[1] != c or out_row_off < 0 or out_row_off + m > o2.shape[0] or ss.numel() < m:
        raise ValueError(f"rmsnorm_rope: rows {out_row_off}..{out_row_off + m} outside the output ({o2.shape[0]} rows)")
    if rope is not None:
        cos, sin, nf = rope
        gh, gw = int(grid[1]), int(grid[2])
    else:
        cos = sin = None
        nf = gh = gw = 0
    check(load().lbw_rmsnorm_rope_dt(ptr(x), ptr(ss), ptr(gamma), m, c, ctypes.c_float(eps), ptr(cos), ptr(sin), nf,
                                     gh, gw, tok0, ptr(o2), o2.stride(0), out_row_off, 1 if rope_bf16 else 0,
                                     stream_of(x.device)), "rmsnorm_rope")
    return out


def qk_rmsnorm_rope(q_raw, ss_q, gamma_q, q_out, k_raw, ss_k, gamma_k, k_out, eps, rope, grid, tok0=0, q_row_off=0,
                    k_row_off=0, rope_bf16=False, _eager=False):
    """rmsnorm_rope of q and k of the same tokens in one launch (lbw_qk_rmsnorm_rope, the reference's
    qk_post.qk_norm_rope): q_out rows q_row_off.., k_out rows k_row_off.. get the normalised, rotated rows.
    rope_bf16: the reference's bf16 rotation (rope.ROPE_DTYPE), else fp32."""
    if _tracing(_eager):
        _op("qk_rmsnorm_rope")(q_raw, ss_q, gamma_q, q_out, k_raw, ss_k, gamma_k, k_out, float(eps), rope[0],
                               rope[1], int(rope[2]), int(grid[1]), int(grid[2]), int(tok0), int(q_row_off),
                               int(k_row_off), bool(rope_bf16))
        return q_out, k_out
    require_cuda(q_raw, ss_q, gamma_q, q_out, k_raw, ss_k, gamma_k, k_out)
    m, c = q_raw.shape
    qo, ko = _rows(q_out), _rows(k_out)
    if k_raw.shape != (m, c) or ss_q.numel() < m or ss_k.numel() < m or qo.shape[1] != c or ko.shape[1] != c:
        raise ValueError("qk_rmsnorm_rope: q and k rows do not match")
    if q_row_off < 0 or q_row_off + m > qo.shape[0] or k_row_off < 0 or k_row_off + m > ko.shape[0]:
        raise ValueError("qk_rmsnorm_rope: rows outside an output")
    cos, sin, nf = rope
    check(load().lbw_qk_rmsnorm_rope_dt(ptr(q_raw), ptr(ss_q), ptr(gamma_q), ptr(qo), qo.stride(0), q_row_off,
                                        ptr(k_raw), ptr(ss_k), ptr(gamma_k), ptr(ko), ko.stride(0), k_row_off, m, c,
                                        ctypes.c_float(eps), ptr(cos), ptr(sin), nf, int(grid[1]), int(grid[2]), tok0,
                                        1 if rope_bf16 else 0, stream_of(q_raw.device)), "qk_rmsnorm_rope")
    return q_out, k_out


MX_FORMATS = {"e4m3": 0, "e5m2": 1, "e2m1": 2}   # lbw_mx_format (include/lbw.h)


def mx_row_bytes(k, fmt="e4m3"):
    """Bytes of one row of k elements: k for the MXFP8 formats, k / 2 for E2M1 (packed nibbles)."""
    return k // 2 if fmt == "e2m1" else k


def mx_quantize(x, dequant=False, data=None, scales=None, fmt="e4m3", _eager=False):
    """x [rows, K] bf16 -> (data uint8 [rows, K] codes ([rows, K / 2] packed for fmt "e2m1"), scales uint8 tiled,
    dequant bf16 or None). fmt: "e4m3" (default), "e5m2" or "e2m1". data / scales: optional output buffers
    (mx_buffers(rows, K, fmt=fmt))."""
    if _tracing(_eager) and not dequant:
        if data is None and scales is None:
            d, sc = _op("mx_quantize")(x, fmt)
            return d, sc, None
        _op("mx_quantize_into")(x, data, scales, fmt)
        return data, scales, None
    require_cuda(x, data, scales)
    _c(x, BF16)
    if fmt not in MX_FORMATS:
        raise ValueError(f"mx_quantize: element format {fmt!r} (one of {sorted(MX_FORMATS)})")
    rows, k = x.shape
    rows_pad = (rows + 127) // 128 * 128
    rb = mx_row_bytes(k, fmt)
    if (data is None) != (scales is None):
        raise ValueError("mx_quantize: give both data and scales, or neither")
    if data is None:
        data = torch.empty(rows, rb, dtype=torch.uint8, device=x.device)
        scales = torch.empty(rows_pad * (k // 32), dtype=torch.uint8, device=x.device)
    elif (data.shape != (rows, rb) or data.dtype != torch.uint8 or not data.is_contiguous()
          or scales.dtype != torch.uint8 or scales.numel() < rows_pad * (k // 32)):
        raise ValueError("mx_quantize: output buffers do not match x")
    deq = torch.empty_like(x) if dequant else None
    check(load().lbw_mx_quantize_fmt(ptr(x), rows, k, MX_FORMATS[fmt], ptr(data), ptr(scales), ptr(deq),
                                     stream_of(x.device)), "mx_quantize")
    return data, scales, deq


def mx_buffers(rows, k, device, fmt="e4m3"):
    """Zeroed MX operand buffers: codes [rows, row bytes] uint8 and tiled scales (rows padded to 128)."""
    rows_pad = (rows + 127) // 128 * 128
    return (torch.zeros(rows, mx_row_bytes(k, fmt), dtype=torch.uint8, device=device),
            torch.zeros(rows_pad * (k // 32), dtype=torch.uint8, device=device))


def _fp8_fmt(fmt, who):
    if fmt not in ("e4m3", "e5m2"):
        raise ValueError(f"{who}: element format {fmt!r} (e4m3 or e5m2)")
    return MX_FORMATS[fmt]


def layernorm_mod_mx(x, eps, scale, shift, data, scales, fmt="e4m3", _eager=False):
    """LN(x) * (1 + scale) + shift -> MX codes (E4M3, or E5M2 with fmt="e5m2") + tiled E8M0 scales."""
    if _tracing(_eager):
        _op("layernorm_mod_mx")(x, float(eps), scale, shift, data, scales, fmt)
        return data, scales
    require_cuda(x, scale, shift, data, scales)
    _c(x, torch.float32)
    m, c = x.shape
    if data.shape != (m, c) or scales.numel() < (m + 127) // 128 * 128 * (c // 32):
        raise ValueError("layernorm_mod_mx: output buffers do not match x")
    check(load().lbw_layernorm_mod_mx_fmt(ptr(x), m, c, ctypes.c_float(eps), ptr(scale), ptr(shift),
                                          _fp8_fmt(fmt, "layernorm_mod_mx"), ptr(data), ptr(scales),
                                          stream_of(x.device)), "layernorm_mod_mx")
    return data, scales


def layernorm_affine_mx(x, eps, weight, bias, data, scales, fmt="e4m3", _eager=False):
    """MXFP8 codes (E4M3, or E5M2 with fmt="e5m2") + tiled scales of LN(x) * weight + bias (norm3 before an MXFP8
    cross_attn.q)."""
    if _tracing(_eager):
        _op("layernorm_affine_mx")(x, float(eps), weight, bias, data, scales, fmt)
        return data, scales
    require_cuda(x, weight, bias, data, scales)
    _c(x, torch.float32), _c(weight, torch.float32), _c(bias, torch.float32)
    m, c = x.shape
    if data.shape != (m, c) or scales.numel() < (m + 127) // 128 * 128 * (c // 32):
        raise ValueError("layernorm_affine_mx: output buffers do not match x")
    check(load().lbw_layernorm_affine_mx_fmt(ptr(x), m, c, ctypes.c_float(eps), ptr(weight), ptr(bias),
                                             _fp8_fmt(fmt, "layernorm_affine_mx"), ptr(data), ptr(scales),
                                             stream_of(x.device)), "layernorm_affine_mx")
    return data, scales


def _mx_check(a, a_s, w, w_s, fmt="e4m3"):
    """(m, n, k) of an MX GEMM, k in elements (a row of E2M1 codes holds k / 2 bytes)."""
    require_cuda(a, a_s, w, w_s)
    m, kb = a.shape
    n = w.shape[0]
    k = kb * 2 if fmt == "e2m1" else kb
    if a.dtype != torch.uint8 or w.dtype != torch.uint8 or w.shape[1] != kb:
        raise ValueError("mx gemm: codes must be uint8 [m, k] and [n, k] (k / 2 bytes per row for e2m1)")
    if a_s.numel() < (m + 127) // 128 * 128 * (k // 32) or w_s.numel() < (n + 127) // 128 * 128 * (k // 32):
        raise ValueError("mx gemm: scale buffers too small")
    return m, n, k


def mx_linear(a, a_s, w, w_s, bias=None, out=None, fmt="e4m3", _eager=False):
    """out [m, n] = bf16(bf16(a w^T) + bias) on the block-scaled GEMM; a, w as mx_quantize(..., fmt=fmt) made them."""
    if _tracing(_eager):
        y = _op("mx_linear")(a, a_s, w, w_s, bias, fmt)
        if out is None:
            return y
        out.copy_(y)
        return out
    if fmt not in MX_FORMATS:
        raise ValueError(f"mx_linear: element format {fmt!r} (one of {sorted(MX_FORMATS)})")
    m, n, k = _mx_check(a, a_s, w, w_s, fmt)
    if out is None:
        out = torch.empty(m, n, dtype=BF16, device=a.device)
    check(load().lbw_mx_linear_fmt(ptr(a), ptr(a_s), ptr(w), ptr(w_s), ptr(bias), m, n, k, MX_FORMATS[fmt], ptr(out),
                                   stream_of(a.device)), "mx_linear")
    return out


def mx_linear_gelu(a, a_s, w, w_s, bias, out, out_scales, fmt="e4m3", _eager=False):
    """FFN-up: GELU(bf16(a w^T) + bias) -> MX codes + scales, operands and output in fmt (e4m3 or e5m2)."""
    if _tracing(_eager):
        _op("mx_linear_gelu")(a, a_s, w, w_s, bias, out, out_scales, fmt)
        return out, out_scales
    m, n, k = _mx_check(a, a_s, w, w_s)
    if out.shape != (m, n) or out.dtype != torch.uint8:
        raise ValueError("mx_linear_gelu: out must be uint8 [m, n]")
    check(load().lbw_mx_linear_gelu_fmt(ptr(a), ptr(a_s), ptr(w), ptr(w_s), ptr(bias), m, n, k,
                                        _fp8_fmt(fmt, "mx_linear_gelu"), ptr(out), ptr(out_scales),
                                        stream_of(a.device)), "mx_linear_gelu")
    return out, out_scales


def mx_linear_residual(a, a_s, w, w_s, bias, x, gate=None, film_scale=None, film_shift=None, fmt="e4m3",
                       _eager=False):
    """x += bf16(bf16(a w^T) + bias) * gate (then the optional FiLM), operands in fmt (e4m3 or e5m2)."""
    if _tracing(_eager):
        _op("mx_linear_residual")(a, a_s, w, w_s, bias, x, gate, film_scale, film_shift, fmt)
        return x
    m, n, k = _mx_check(a, a_s, w, w_s)
    require_cuda(x, gate, film_scale, film_shift)
    if x.shape != (m, n) or x.dtype != torch.float32:
        raise ValueError("mx_linear_residual: x must be fp32 [m, n]")
    if film_scale is None and film_shift is None:
        check(load().lbw_mx_linear_residual_fmt(ptr(a), ptr(a_s), ptr(w), ptr(w_s), ptr(bias), m, n, k,
                                                _fp8_fmt(fmt, "mx_linear_residual"), ptr(x), ptr(gate),
                                                stream_of(a.device)), "mx_linear_residual")
        return x

    for t in (film_scale, film_shift):
        if t is None or t.shape != (m, n) or t.dtype != BF16 or not t.is_contiguous():
            raise ValueError("mx_linear_residual: FiLM tensors must both be contiguous bf16 [m, n]")
    check(load().lbw_mx_linear_residual_film_fmt(ptr(a), ptr(a_s), ptr(w), ptr(w_s), ptr(bias), m, n, k,
                                                 _fp8_fmt(fmt, "mx_linear_residual"), ptr(x), ptr(gate),
                                                 ptr(film_scale), ptr(film_shift), stream_of(a.device)),
          "mx_linear_residual_film")
    return x


def mx_qkv_proj(hq, hs, w_qkv, w_qkv_s, b_qkv, q_raw, k_raw, ss_q, ss_k, v_out, v_row_off=0, fmt="e4m3"):
    """MXFP8 counterpart of qkv_proj: hq/hs the MXFP8 operand of the normed rows, w_qkv/w_qkv_s of [Wq; Wk; Wv];
    fmt: the codes' element format (e4m3 or e5m2)."""
    m, n, c = _mx_check(hq, hs, w_qkv, w_qkv_s)
    require_cuda(b_qkv, q_raw, k_raw, ss_q, ss_k, v_out)
    v2 = _rows(v_out)
    if n != 3 * c or q_raw.shape != (m, c) or k_raw.shape != (m, c) or ss_q.numel() < m or ss_k.numel() < m:
        raise ValueError("mx_qkv_proj: shape mismatch")
    if v2.shape[1] != c or v_row_off < 0 or v_row_off + m > v2.shape[0]:
        raise ValueError(f"mx_qkv_proj: rows {v_row_off}..{v_row_off + m} outside the V destination "
                         f"({v2.shape[0]} rows)")
    check(load().lbw_mx_qkv_proj_fmt(ptr(hq), ptr(hs), ptr(w_qkv), ptr(w_qkv_s), ptr(b_qkv), m, c,
                                     _fp8_fmt(fmt, "mx_qkv_proj"), ptr(q_raw), ptr(k_raw), ptr(ss_q), ptr(ss_k),
                                     ptr(v2), v2.stride(0), v_row_off, stream_of(hq.device)), "mx_qkv_proj")


def mx_linear_rowss(a, a_s, w, w_s, bias, out, ss, fmt="e4m3"):
    m, n, k = _mx_check(a, a_s, w, w_s)
    require_cuda(bias, out, ss)
    if out.shape != (m, n) or out.dtype != BF16 or not out.is_contiguous() or ss.numel() < m:
        raise ValueError("mx_linear_rowss: shape mismatch")
    check(load().lbw_mx_linear_rowss_fmt(ptr(a), ptr(a_s), ptr(w), ptr(w_s), ptr(bias), m, n, k,
                                         _fp8_fmt(fmt, "mx_linear_rowss"), ptr(out), ptr(ss), stream_of(a.device)),
          "mx_linear_rowss")
    return out


def mx_linear_act(a, a_s, w, w_s, bias=None, addend=None, silu=False, out=None, fmt="e4m3"):
    """MXFP8 counterpart of linear_act (camera-FiLM MLP layers); fmt: e4m3 or e5m2."""
    m, n, k = _mx_check(a, a_s, w, w_s)
    require_cuda(bias, addend, out)
    if addend is not None and (addend.shape != (m, n) or addend.dtype != BF16 or not addend.is_contiguous()):
        raise ValueError("mx_linear_act: addend must be contiguous bf16 [m, n]")
    if out is None:
        out = torch.empty(m, n, dtype=BF16, device=a.device)
    check(load().lbw_mx_linear_act_fmt(ptr(a), ptr(a_s), ptr(w), ptr(w_s), ptr(bias), ptr(addend), int(bool(silu)), m,
                                       n, k, _fp8_fmt(fmt, "mx_linear_act"), ptr(out), stream_of(a.device)),
          "mx_linear_act")
    return out


# ---------------------------------------------------------------------------------------------- VAE decoder
def _avail(t):
    """Elements addressable from t.data_ptr() to the end of its storage (bounds of strided views)."""
    return (t.untyped_storage().nbytes() - t.storage_offset() * t.element_size()) // t.element_size()


def vae_conv(x, in_rows, c_in, w, bias, c_out, k, frames, h, wd, out, residual=None):
    """Causal conv over padded frames (lbw_vae_conv); k = (kt, kh, kw)."""
    require_cuda(x, w, bias, out, residual)
    kt, kh, kw = k
    P = (h + 2) * (wd + 2)
    ck = (c_in + 63) // 64 * 64             # K-space channels per tap (zero weights past c_in)
    if x.numel() < in_rows * c_in or w.numel() != c_out * kt * kh * kw * ck or out.numel() < frames * P * c_out:
        raise ValueError("vae_conv: buffer sizes do not match the convolution")
    if residual is not None and residual.numel() < frames * P * c_out:
        raise ValueError("vae_conv: residual smaller than the output")
    check(load().lbw_vae_conv(ptr(x), in_rows, c_in, ptr(w), ptr(bias), c_out, kt, kh, kw, frames, h, wd,
                              ptr(residual), ptr(out), stream_of(x.device)), "vae_conv")
    return out


def vae_conv_rms(x, in_rows, c_in, w, bias, c_out, k, frames, h, wd, gamma, c_real, out):
    """vae_conv fused with the RMS_norm + SiLU of its output rows (c_out <= 256)."""
    require_cuda(x, w, bias, gamma, out)
    kt, kh, kw = k
    P = (h + 2) * (wd + 2)
    ck = (c_in + 63) // 64 * 64
    if x.numel() < in_rows * c_in or w.numel() != c_out * kt * kh * kw * ck or out.numel() < frames * P * c_out:
        raise ValueError("vae_conv_rms: buffer sizes do not match the convolution")
    if gamma.dtype != torch.float32 or gamma.numel() < c_out:
        raise ValueError("vae_conv_rms: gamma must be fp32 [c_out]")
    check(load().lbw_vae_conv_rms(ptr(x), in_rows, c_in, ptr(w), ptr(bias), c_out, kt, kh, kw, frames, h, wd,
                                  ptr(gamma), c_real, ptr(out), stream_of(x.device)), "vae_conv_rms")
    return out


def vae_rms_silu(x, rows, c, c_real, gamma, silu, out):
    require_cuda(x, gamma, out)
    if x.numel() < rows * c or out.numel() < rows * c or gamma.numel() < c or gamma.dtype != torch.float32:
        raise ValueError("vae_rms_silu: buffer sizes")
    check(load().lbw_vae_rms_silu(ptr(x), rows, c, c_real, ptr(gamma), int(bool(silu)), ptr(out),
                                  stream_of(x.device)), "vae_rms_silu")
    return out


def vae_upsample2x(x, frames, h, w, c, out):
    require_cuda(x, out)
    if x.numel() < frames * (h + 2) * (w + 2) * c or out.numel() < frames * (2 * h + 2) * (2 * w + 2) * c:
        raise ValueError("vae_upsample2x: buffer sizes")
    check(load().lbw_vae_upsample2x(ptr(x), frames, h, w, c, ptr(out), stream_of(x.device)), "vae_upsample2x")
    return out


def vae_time_interleave(x, frames, frame_rows, c, out):
    require_cuda(x, out)
    if x.numel() < frames * frame_rows * 2 * c or out.numel() < 2 * frames * frame_rows * c:
        raise ValueError("vae_time_interleave: buffer sizes")
    check(load().lbw_vae_time_interleave(ptr(x), frames, frame_rows, c, ptr(out), stream_of(x.device)),
          "vae_time_interleave")
    return out


def vae_gather(x, frames, h, w, c, out):
    require_cuda(x, out)
    if x.numel() < frames * (h + 2) * (w + 2) * c or out.numel() < frames * h * w * c:
        raise ValueError("vae_gather: buffer sizes")
    check(load().lbw_vae_gather(ptr(x), frames, h, w, c, ptr(out), stream_of(x.device)), "vae_gather")
    return out


def vae_scatter_add(y, resid, frames, h, w, c, out):
    require_cuda(y, resid, out)
    P = (h + 2) * (w + 2)
    if y.numel() < frames * h * w * c or resid.numel() < frames * P * c or out.numel() < frames * P * c:
        raise ValueError("vae_scatter_add: buffer sizes")
    check(load().lbw_vae_scatter_add(ptr(y), ptr(resid), frames, h, w, c, ptr(out), stream_of(y.device)),
          "vae_scatter_add")
    return out


def gemm_f32(a, lda, w, ldw, out, ldo, m, n, k):
    """out[m, n] (fp32) = a[m, :k] w[n, :k]^T with explicit row strides."""
    require_cuda(a, w, out)
    if out.dtype != torch.float32 or out.numel() < (m - 1) * ldo + n:
        raise ValueError("gemm_f32: output")
    if _avail(a) < (m - 1) * lda + k or _avail(w) < (n - 1) * ldw + k:
        raise ValueError("gemm_f32: operand sizes")
    check(load().lbw_gemm_f32(ptr(a), lda, ptr(w), ldw, ptr(out), ldo, m, n, k, stream_of(a.device)), "gemm_f32")
    return out


def softmax_rows(s, rows, n, n_pad, scale, p):
    require_cuda(s, p)
    lds, ldp = s.stride(0), p.stride(0)
    if s.shape[0] < rows or p.shape[0] < rows or s.shape[1] < n or p.shape[1] < n_pad:
        raise ValueError("softmax_rows: shapes")
    check(load().lbw_softmax_rows(ptr(s), lds, rows, n, n_pad, ctypes.c_float(scale), ptr(p), ldp,
                                  stream_of(s.device)), "softmax_rows")
    return p


def transpose_bf16(x, ldx, rows, cols, out, ldo):
    require_cuda(x, out)
    if _avail(x) < (rows - 1) * ldx + cols or _avail(out) < (cols - 1) * ldo + rows:
        raise ValueError("transpose_bf16: sizes")
    check(load().lbw_transpose_bf16(ptr(x), ldx, rows, cols, ptr(out), ldo, stream_of(x.device)), "transpose_bf16")
    return out
