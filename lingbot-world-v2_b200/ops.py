"""The C-ABI kernels as PyTorch custom operators: torch.ops.lbw.*.

The reference runs its block stack inside compiled graphs (wan/modules/model_fast.py:3808-3826: groups of
blocks under torch.compile(fullgraph=True)). A plain ctypes call is opaque to the compiler, so every kernel
the drop-in block launches is also registered here with torch.library: each operator declares the tensors it
writes in place (the block's scratch, the fp32 residual, the destination KV-cache chunk) and has a fake
implementation that only describes its outputs, so the compiler traces the block forward into one graph and
runs the real kernels at execution. The torch wrappers of lbw_b200.kernels call these operators while a
graph is being traced and the C ABI directly otherwise, so eager code pays no dispatcher cost.
"""
from typing import List, Optional

import torch

from . import kernels as K

BF16 = torch.bfloat16


@torch.library.custom_op("lbw::chunk_attention", mutates_args=("out",))
def chunk_attention(q: torch.Tensor, k_chunks: List[torch.Tensor], v_chunks: List[torch.Tensor],
                    key_bias: Optional[torch.Tensor], scale: float, out: torch.Tensor) -> None:
    """softmax(q kᵀ * scale + bias) v over the concatenated KV chunks (attention.exact_attention_chunks)."""
    K.chunk_attention(q, k_chunks, v_chunks, key_bias=key_bias, out=out, softmax_scale=scale, _eager=True)


@chunk_attention.register_fake
def _(q, k_chunks, v_chunks, key_bias, scale, out):
    return None


@torch.library.custom_op("lbw::chunk_attention_partial", mutates_args=("part_o", "part_ml"))
def chunk_attention_partial(q: torch.Tensor, k_chunks: List[torch.Tensor], v_chunks: List[torch.Tensor],
                            n_splits: int, part_o: torch.Tensor, part_ml: torch.Tensor, slot0: int,
                            key_bias: Optional[torch.Tensor], scale: float) -> None:
    K.chunk_attention_partial(q, k_chunks, v_chunks, n_splits, part_o, part_ml, slot0, key_bias=key_bias,
                              softmax_scale=scale, _eager=True)


@chunk_attention_partial.register_fake
def _(q, k_chunks, v_chunks, n_splits, part_o, part_ml, slot0, key_bias, scale):
    return None


@torch.library.custom_op("lbw::chunk_attention_tail", mutates_args=("out", "part_o", "part_ml"))
def chunk_attention_tail(q: torch.Tensor, k_chunks: List[torch.Tensor], v_chunks: List[torch.Tensor],
                         key_bias: Optional[torch.Tensor], scale: float, out: torch.Tensor,
                         part_o: Optional[torch.Tensor], part_ml: Optional[torch.Tensor], pieces: int) -> None:
    """chunk_attention with the windows past the last full wave cut into key ranges and merged (lbw.h)."""
    ws = (part_o, part_ml) if part_o is not None else None
    K.chunk_attention_tail(q, k_chunks, v_chunks, ws, key_bias=key_bias, out=out, pieces=pieces, softmax_scale=scale,
                           _eager=True)


@chunk_attention_tail.register_fake
def _(q, k_chunks, v_chunks, key_bias, scale, out, part_o, part_ml, pieces):
    return None


@torch.library.custom_op("lbw::attention_merge", mutates_args=("out",))
def attention_merge(part_o: torch.Tensor, part_ml: torch.Tensor, n_slots: int, out: torch.Tensor) -> None:
    K.attention_merge(part_o, part_ml, n_slots, out, _eager=True)


@attention_merge.register_fake
def _(part_o, part_ml, n_slots, out):
    return None


@torch.library.custom_op("lbw::layernorm_mod", mutates_args=("out",))
def layernorm_mod(x: torch.Tensor, eps: float, out: torch.Tensor, scale: Optional[torch.Tensor],
                  shift: Optional[torch.Tensor], weight: Optional[torch.Tensor], bias: Optional[torch.Tensor],
                  mx_qdq: bool) -> None:
    K.layernorm_mod(x, eps, out, scale=scale, shift=shift, weight=weight, bias=bias, mx_qdq=mx_qdq, _eager=True)


@layernorm_mod.register_fake
def _(x, eps, out, scale, shift, weight, bias, mx_qdq):
    return None


@torch.library.custom_op("lbw::layernorm_mod_mx", mutates_args=("data", "scales"))
def layernorm_mod_mx(x: torch.Tensor, eps: float, scale: torch.Tensor, shift: torch.Tensor, data: torch.Tensor,
                     scales: torch.Tensor, fmt: str) -> None:
    K.layernorm_mod_mx(x, eps, scale, shift, data, scales, fmt=fmt, _eager=True)


@layernorm_mod_mx.register_fake
def _(x, eps, scale, shift, data, scales, fmt):
    return None


@torch.library.custom_op("lbw::layernorm_affine_mx", mutates_args=("data", "scales"))
def layernorm_affine_mx(x: torch.Tensor, eps: float, weight: torch.Tensor, bias: torch.Tensor, data: torch.Tensor,
                        scales: torch.Tensor, fmt: str) -> None:
    K.layernorm_affine_mx(x, eps, weight, bias, data, scales, fmt=fmt, _eager=True)


@layernorm_affine_mx.register_fake
def _(x, eps, weight, bias, data, scales, fmt):
    return None


@torch.library.custom_op("lbw::qkv_proj", mutates_args=("q_raw", "k_raw", "ss_q", "ss_k", "v_out"))
def qkv_proj(h: torch.Tensor, w_qkv: torch.Tensor, b_qkv: torch.Tensor, q_raw: torch.Tensor, k_raw: torch.Tensor,
             ss_q: torch.Tensor, ss_k: torch.Tensor, v_out: torch.Tensor, v_row_off: int) -> None:
    K.qkv_proj(h, w_qkv, b_qkv, q_raw, k_raw, ss_q, ss_k, v_out, v_row_off=v_row_off, _eager=True)


@qkv_proj.register_fake
def _(h, w_qkv, b_qkv, q_raw, k_raw, ss_q, ss_k, v_out, v_row_off):
    return None


@torch.library.custom_op("lbw::rmsnorm_rope", mutates_args=("out",))
def rmsnorm_rope(x: torch.Tensor, ss: torch.Tensor, gamma: torch.Tensor, eps: float, out: torch.Tensor,
                 cos: Optional[torch.Tensor], sin: Optional[torch.Tensor], n_frames: int, grid_h: int, grid_w: int,
                 tok0: int, out_row_off: int, rope_bf16: bool) -> None:
    rope = (cos, sin, n_frames) if cos is not None else None
    grid = (n_frames, grid_h, grid_w) if cos is not None else None
    K.rmsnorm_rope(x, ss, gamma, eps, out, rope=rope, grid=grid, tok0=tok0, out_row_off=out_row_off,
                   rope_bf16=rope_bf16, _eager=True)


@rmsnorm_rope.register_fake
def _(x, ss, gamma, eps, out, cos, sin, n_frames, grid_h, grid_w, tok0, out_row_off, rope_bf16):
    return None


@torch.library.custom_op("lbw::qk_rmsnorm_rope", mutates_args=("q_out", "k_out"))
def qk_rmsnorm_rope(q_raw: torch.Tensor, ss_q: torch.Tensor, gamma_q: torch.Tensor, q_out: torch.Tensor,
                    k_raw: torch.Tensor, ss_k: torch.Tensor, gamma_k: torch.Tensor, k_out: torch.Tensor, eps: float,
                    cos: torch.Tensor, sin: torch.Tensor, n_frames: int, grid_h: int, grid_w: int, tok0: int,
                    q_row_off: int, k_row_off: int, rope_bf16: bool) -> None:
    """q and k RMSNorm + RoPE in one launch (kernels/qk_post.py qk_norm_rope)."""
    K.qk_rmsnorm_rope(q_raw, ss_q, gamma_q, q_out, k_raw, ss_k, gamma_k, k_out, eps, (cos, sin, n_frames),
                      (n_frames, grid_h, grid_w), tok0=tok0, q_row_off=q_row_off, k_row_off=k_row_off,
                      rope_bf16=rope_bf16, _eager=True)


@qk_rmsnorm_rope.register_fake
def _(q_raw, ss_q, gamma_q, q_out, k_raw, ss_k, gamma_k, k_out, eps, cos, sin, n_frames, grid_h, grid_w, tok0,
      q_row_off, k_row_off, rope_bf16):
    return None


@torch.library.custom_op("lbw::linear_residual", mutates_args=("x",))
def linear_residual(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], x: torch.Tensor,
                    gate: Optional[torch.Tensor], film_scale: Optional[torch.Tensor],
                    film_shift: Optional[torch.Tensor]) -> None:
    K.linear_residual(a, w, bias, x, gate=gate, film_scale=film_scale, film_shift=film_shift, _eager=True)


@linear_residual.register_fake
def _(a, w, bias, x, gate, film_scale, film_shift):
    return None


@torch.library.custom_op("lbw::linear_rowss", mutates_args=("out", "ss"))
def linear_rowss(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], out: torch.Tensor,
                 ss: torch.Tensor) -> None:
    K.linear_rowss(a, w, bias, out, ss, _eager=True)


@linear_rowss.register_fake
def _(a, w, bias, out, ss):
    return None


@torch.library.custom_op("lbw::linear_gelu", mutates_args=("out",))
def linear_gelu(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, out: torch.Tensor, mx_qdq: bool) -> None:
    K.linear_gelu(a, w, bias, out, mx_qdq, _eager=True)


@linear_gelu.register_fake
def _(a, w, bias, out, mx_qdq):
    return None


@torch.library.custom_op("lbw::mx_linear_gelu", mutates_args=("out", "out_scales"))
def mx_linear_gelu(a: torch.Tensor, a_s: torch.Tensor, w: torch.Tensor, w_s: torch.Tensor, bias: torch.Tensor,
                   out: torch.Tensor, out_scales: torch.Tensor, fmt: str) -> None:
    K.mx_linear_gelu(a, a_s, w, w_s, bias, out, out_scales, fmt=fmt, _eager=True)


@mx_linear_gelu.register_fake
def _(a, a_s, w, w_s, bias, out, out_scales, fmt):
    return None


@torch.library.custom_op("lbw::mx_linear_residual", mutates_args=("x",))
def mx_linear_residual(a: torch.Tensor, a_s: torch.Tensor, w: torch.Tensor, w_s: torch.Tensor,
                       bias: Optional[torch.Tensor], x: torch.Tensor, gate: Optional[torch.Tensor],
                       film_scale: Optional[torch.Tensor], film_shift: Optional[torch.Tensor], fmt: str) -> None:
    K.mx_linear_residual(a, a_s, w, w_s, bias, x, gate=gate, film_scale=film_scale, film_shift=film_shift, fmt=fmt,
                         _eager=True)


@mx_linear_residual.register_fake
def _(a, a_s, w, w_s, bias, x, gate, film_scale, film_shift, fmt):
    return None


@torch.library.custom_op("lbw::mx_quantize_into", mutates_args=("data", "scales"))
def mx_quantize_into(x: torch.Tensor, data: torch.Tensor, scales: torch.Tensor, fmt: str) -> None:
    """x -> MX codes + tiled E8M0 scales in the given buffers (ffn_mx.prequantize_weight / the activation
    quantisation of ffn_mx.mm)."""
    K.mx_quantize(x, data=data, scales=scales, fmt=fmt, _eager=True)


@mx_quantize_into.register_fake
def _(x, data, scales, fmt):
    return None


@torch.library.custom_op("lbw::mx_quantize", mutates_args=())
def mx_quantize(x: torch.Tensor, fmt: str) -> List[torch.Tensor]:
    """x [rows, K] bf16 -> [codes, tiled scales] (a new pair)."""
    d, s, _ = K.mx_quantize(x, fmt=fmt, _eager=True)
    return [d, s]


@mx_quantize.register_fake
def _(x, fmt):
    rows, k = x.shape
    rows_pad = (rows + 127) // 128 * 128
    return [x.new_empty((rows, K.mx_row_bytes(k, fmt)), dtype=torch.uint8),
            x.new_empty((rows_pad * (k // 32),), dtype=torch.uint8)]


@torch.library.custom_op("lbw::mx_linear", mutates_args=())
def mx_linear(a: torch.Tensor, a_s: torch.Tensor, w: torch.Tensor, w_s: torch.Tensor, bias: Optional[torch.Tensor],
              fmt: str) -> torch.Tensor:
    """bf16(bf16(a wᵀ) + bias) on the block-scaled GEMM (ffn_mx.mm)."""
    return K.mx_linear(a, a_s, w, w_s, bias, fmt=fmt, _eager=True)


@mx_linear.register_fake
def _(a, a_s, w, w_s, bias, fmt):
    return a.new_empty((a.shape[0], w.shape[0]), dtype=BF16)


OPS = ("chunk_attention", "chunk_attention_partial", "chunk_attention_tail", "attention_merge", "layernorm_mod", "layernorm_mod_mx",
       "layernorm_affine_mx", "qkv_proj", "rmsnorm_rope", "qk_rmsnorm_rope", "linear_residual", "linear_rowss", "linear_gelu",
       "mx_linear_gelu", "mx_linear_residual", "mx_quantize_into", "mx_quantize", "mx_linear")
