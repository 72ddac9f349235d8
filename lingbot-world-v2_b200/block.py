"""Drop-in CausalWanAttentionBlock for B200.

Same constructor, parameter names (state_dict keys) and forward signature as the reference's
wan/modules/model_fast.py:2837-3116 CausalWanAttentionBlock, for the path the causal-fast pipeline
runs: the chunked KV cache (kv_chunks=(k_chunks, v_chunks), destination LAST, layout
[1, chunk_tokens, n, 128]), hoisted camera FiLM (dit_cond_dict={"cam_film": (scale, shift)}), the
cached text cross-attention (crossattn_cache={"k", "v", "is_init"}), optional cross_dedup, and the
MXFP8 FFN (ffn_mx=True, LINGBOT_FFN_MX) or the bf16 FFN. lin_mx=True (LINGBOT_LIN_MX, model_fast.py:1266-1269,
:1442-1494) puts the other block Linears on the MXFP8 GEMM too, except those named in lin_mx_skip
(LINGBOT_LIN_MX_SKIP): their inputs are quantised by the producing LayerNorm kernel or by mx_quantize.

One forward = 13 kernels of liblbw.so on the current stream:
  layernorm_mod(norm1 + adaLN) -> qkv_proj (v straight into the destination chunk) ->
  qk_rmsnorm_rope(q, and k into the destination chunk, one launch) -> [sequence-parallel K/V all-gather]
  -> chunk_attention -> linear_residual(o-proj, gate e2, FiLM) -> layernorm(norm3 affine) ->
  linear_rowss(cross q) -> rmsnorm(cross q) -> chunk_attention(cross, optional dedup bias) ->
  linear_residual(cross o) -> layernorm_mod(norm2 + adaLN, MX QDQ) -> linear_gelu(ffn.0 + GELU, MX QDQ)
  -> linear_residual(ffn.2, gate e5)
(with the MXFP8 FFN the last three are layernorm_mod_mx -> mx_linear_gelu -> mx_linear_residual; lin_mx adds
an mx_quantize of the attention output before each of the two o-projections).
The fp32 residual is updated in place by the GEMM epilogues.
"""

import torch
import torch.nn as nn

from . import ffn_mx as _ffn_mx
from . import kernels, ops, rope, sp  # noqa: F401  (ops registers the kernels as torch.ops.lbw.*)
from .attention import cross_dedup_bias

BF16 = torch.bfloat16
HEAD_DIM = 128
# model_fast.py:1304-1306 (_MX_LIN_NAMES): the Linears LINGBOT_LIN_MX quantises besides the FFN
MX_LINEAR_NAMES = ("self_attn.q", "self_attn.k", "self_attn.v", "self_attn.o",
                   "cross_attn.q", "cross_attn.k", "cross_attn.v", "cross_attn.o",
                   "cam_injector_layer1", "cam_injector_layer2", "cam_scale_layer", "cam_shift_layer")
# packed-weight key of each (q|k|v share the fused GEMM)
_MX_KEYS = {"self_attn.o": "wo", "cross_attn.q": "wcq", "cross_attn.k": "wck", "cross_attn.v": "wcv",
            "cross_attn.o": "wco", "cam_injector_layer1": "wc1", "cam_injector_layer2": "wc2",
            "cam_scale_layer": "wcs", "cam_shift_layer": "wcsh"}


class _RMSNormParam(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))


class _AttnParams(nn.Module):
    """q/k/v/o Linears and the q/k RMSNorm weights (WanSelfAttention / WanCrossAttention layout)."""

    def __init__(self, dim, num_heads, qk_norm=True, eps=1e-6):
        super().__init__()
        self.dim, self.num_heads, self.head_dim, self.eps = dim, num_heads, dim // num_heads, eps
        self.qk_norm = qk_norm
        self.q, self.k, self.v, self.o = (nn.Linear(dim, dim) for _ in range(4))
        self.norm_q = _RMSNormParam(dim) if qk_norm else nn.Identity()
        self.norm_k = _RMSNormParam(dim) if qk_norm else nn.Identity()


def _event():
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev


class Workspace:
    """Scratch of one block forward over `rows` local query tokens; shared by all blocks of a stack."""

    def __init__(self, rows, dim, ffn_dim, device):
        self.rows, self.dim, self.ffn_dim = rows, dim, ffn_dim
        mk = lambda *s, dt=BF16: torch.empty(*s, dtype=dt, device=device)  # noqa: E731
        self.h = mk(rows, dim)
        self.q_raw = mk(rows, dim)
        self.k_raw = mk(rows, dim)
        # row sums of squares of q and k (two tensors: an operator may not write two views of one)
        self.ss_q = mk(rows, dt=torch.float32)
        self.ss_k = mk(rows, dt=torch.float32)
        self.q = mk(rows, dim)
        self.attn = mk(rows, dim)
        self.u = mk(rows, ffn_dim)
        # MXFP8 operands of the FFN: codes + tiled E8M0 scales (rows padded to 128)
        self.hq, self.hs = kernels.mx_buffers(rows, dim, device)
        self.uq, self.us = kernels.mx_buffers(rows, ffn_dim, device)

    def new_kv(self, chunk_rows):
        """Scratch K and V of the new chunk [chunk_rows, dim] bf16 for kv_write=False (the cache slot is left as it
        is), allocated on first use."""
        if getattr(self, "_new_kv", None) is None or self._new_kv[0].shape[0] != chunk_rows:
            self._new_kv = (torch.empty(chunk_rows, self.dim, dtype=BF16, device=self.h.device),
                            torch.empty(chunk_rows, self.dim, dtype=BF16, device=self.h.device))
        return self._new_kv

    def attn_tail(self, heads, chunk_rows):
        """(workspace, pieces) of the self-attention's tail schedule over these key chunks (workspace None when no
        window is cut), planned once per key-chunk shape."""
        if getattr(self, "_tail", None) is None:
            self._tail = {}
        key = (heads, tuple(chunk_rows))
        hit = self._tail.get(key)
        if hit is None:
            dev = self.h.device
            _, pieces = kernels.attention_tail_plan(self.rows, heads, chunk_rows, dev)
            hit = self._tail[key] = (kernels.attention_tail_workspace(self.rows, heads, chunk_rows, dev, pieces), pieces)
        return hit

    def fits(self, rows, dim, ffn_dim, device):
        return (self.rows, self.dim, self.ffn_dim) == (rows, dim, ffn_dim) and self.h.device == device


class CausalWanAttentionBlock(nn.Module):
    def __init__(self, dim, ffn_dim, num_heads, local_attn_size=-1, sink_size=0, qk_norm=True,
                 cross_attn_norm=False, eps=1e-6, ffn_mx=True, cross_dedup=0, mx_pipe="mxf8", lin_mx=False,
                 lin_mx_skip=(), mx_fp8=None):
        """mx_fp8: element format of the MX FFN, "float8_e4m3fn" or "float8_e5m2" (the reference's LINGBOT_MX_FP8,
        kernels/ffn_mx.py:8,18); None takes LINGBOT_MX_FP8 as lbw_b200.ffn_mx read it at import (default E4M3)."""
        super().__init__()
        if dim % num_heads or dim // num_heads != HEAD_DIM:
            raise ValueError("the B200 kernels are built for head_dim 128")
        if not qk_norm:
            raise ValueError("the B200 path fuses the q/k RMSNorm; qk_norm=False is not supported")
        self.dim, self.ffn_dim, self.num_heads = dim, ffn_dim, num_heads
        self.local_attn_size, self.qk_norm, self.cross_attn_norm, self.eps = local_attn_size, qk_norm, cross_attn_norm, eps
        self.ffn_mx = bool(ffn_mx)
        if mx_pipe not in ("mxf8", "bf16"):
            raise ValueError("mx_pipe is 'mxf8' (tcgen05 block-scaled MMA) or 'bf16' (MX values on the bf16 pipe)")
        self.mx_pipe = mx_pipe
        skip = tuple(lin_mx_skip or ())
        unknown = [n for n in skip if n not in MX_LINEAR_NAMES]
        if unknown:
            raise ValueError(f"lin_mx_skip names no block Linear: {unknown} (known: {MX_LINEAR_NAMES})")
        self.lin_mx = bool(lin_mx)
        self.mx_linears = frozenset(n for n in MX_LINEAR_NAMES if n not in skip) if self.lin_mx else frozenset()
        qkv = {"self_attn.q", "self_attn.k", "self_attn.v"} & self.mx_linears
        if qkv and len(qkv) != 3:
            raise ValueError("self_attn.q/k/v share one fused GEMM: lin_mx_skip must name all three or none")
        if self.lin_mx:
            if mx_pipe != "mxf8":
                raise ValueError("lin_mx runs on the block-scaled tcgen05 GEMM (mx_pipe='mxf8')")
            self.ffn_mx = True   # LINGBOT_LIN_MX implies LINGBOT_FFN_MX (model_fast.py:1270)
        fp8 = mx_fp8 or _ffn_mx.FP8
        if fp8 not in _ffn_mx._FMT_OF_DTYPE:
            raise ValueError(f"mx_fp8={fp8!r}: expected one of {sorted(_ffn_mx._FMT_OF_DTYPE)}")
        self.mx_fmt = _ffn_mx._FMT_OF_DTYPE[fp8]
        if self.mx_fmt != "e4m3" and self.ffn_mx and mx_pipe != "mxf8":
            raise ValueError("float8_e5m2 runs on the block-scaled GEMM (mx_pipe='mxf8'); the bf16-pipe variant "
                             "takes E4M3 only")
        self.cross_dedup = int(cross_dedup)
        self.norm1 = nn.Identity()
        self.self_attn = _AttnParams(dim, num_heads, qk_norm, eps)
        self.norm3 = nn.LayerNorm(dim, eps, elementwise_affine=True) if cross_attn_norm else nn.Identity()
        self.cross_attn = _AttnParams(dim, num_heads, qk_norm, eps)
        self.norm2 = nn.Identity()
        self.ffn = nn.Sequential(nn.Linear(dim, ffn_dim), nn.GELU(approximate="tanh"), nn.Linear(ffn_dim, dim))
        self.modulation = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)
        self.cam_injector_layer1 = nn.Linear(dim, dim)
        self.cam_injector_layer2 = nn.Linear(dim, dim)
        self.cam_scale_layer = nn.Linear(dim, dim)
        self.cam_shift_layer = nn.Linear(dim, dim)
        self._packed = None
        self._ws = None

    # ------------------------------------------------------------------ weights
    @torch.no_grad()
    def prepare(self, free_sources=False, with_cam=True):
        """Pack/convert the weights the kernels read (once; call again after changing weights). with_cam keeps
        the camera-FiLM MLP weights for cam_film()."""
        if getattr(self, "_sources_freed", False):
            raise ValueError("prepare(free_sources=True) already released the source weights")
        sa, ca = self.self_attn, self.cross_attn
        dev = sa.q.weight.device
        if dev.type != "cuda":
            raise ValueError("move the block to a CUDA device before the forward")
        b = lambda t: t.detach().to(BF16).contiguous()  # noqa: E731
        mx = self.mx_linears
        pk = {}
        wqkv = torch.cat([b(sa.q.weight), b(sa.k.weight), b(sa.v.weight)]).contiguous()
        if "self_attn.q" in mx:
            # quantised per row along K, so the fused [Wq; Wk; Wv] codes equal the three quantised separately
            pk["wqkv_mx"] = kernels.mx_quantize(wqkv, fmt=self.mx_fmt)[:2]
        else:
            pk["wqkv"] = wqkv
        pk["bqkv"] = torch.cat([b(sa.q.bias), b(sa.k.bias), b(sa.v.bias)]).contiguous()
        pk["gq"], pk["gk"] = b(sa.norm_q.weight), b(sa.norm_k.weight)
        pk["gcq"], pk["gck"] = b(ca.norm_q.weight), b(ca.norm_k.weight)
        for key, lin in (("o", sa.o), ("cq", ca.q), ("ck", ca.k), ("cv", ca.v), ("co", ca.o)):
            self._pack_linear(pk, key, lin, b)
        if self.cross_attn_norm:
            pk["n3w"] = self.norm3.weight.detach().float().contiguous()
            pk["n3b"] = self.norm3.bias.detach().float().contiguous()
        pk["mod"] = self.modulation.detach().float().reshape(6, self.dim).contiguous()
        w1, w2 = b(self.ffn[0].weight), b(self.ffn[2].weight)
        if self.ffn_mx and self.mx_pipe == "mxf8":
            # MXFP8 weights: E4M3 (or E5M2) codes + E8M0 scales read by the block-scaled tcgen05 GEMM
            pk["w1_mx"] = kernels.mx_quantize(w1, fmt=self.mx_fmt)[:2]
            pk["w2_mx"] = kernels.mx_quantize(w2, fmt=self.mx_fmt)[:2]
        elif self.ffn_mx:
            # bf16-pipe variant: the GEMM reads the exact bf16 dequantisation of the MXFP8 weights
            pk["w1"] = kernels.mx_quantize(w1, dequant=True)[2]
            pk["w2"] = kernels.mx_quantize(w2, dequant=True)[2]
        else:
            pk["w1"], pk["w2"] = w1, w2
        pk["b1"], pk["b2"] = b(self.ffn[0].bias), b(self.ffn[2].bias)
        if with_cam:
            for key, lin in (("c1", self.cam_injector_layer1), ("c2", self.cam_injector_layer2),
                             ("cs", self.cam_scale_layer), ("csh", self.cam_shift_layer)):
                self._pack_linear(pk, key, lin, b)
        self._packed = pk
        if free_sources:
            # Only the packed copies serve the forward from here on (the reference frees its bf16 FFN
            # weights the same way after MX quantisation, model_fast.py:1574-1581).
            for lin in (sa.q, sa.k, sa.v, sa.o, ca.q, ca.k, ca.v, ca.o, self.ffn[0], self.ffn[2],
                        self.cam_injector_layer1, self.cam_injector_layer2, self.cam_scale_layer,
                        self.cam_shift_layer):
                lin.weight = nn.Parameter(torch.empty(0, dtype=lin.weight.dtype, device=dev), requires_grad=False)
            self._sources_freed = True
        return pk

    def _mx_name(self, key):
        return next(n for n, k in _MX_KEYS.items() if k == "w" + key)

    def _pack_linear(self, pk, key, lin, b):
        """pk["w" + key] bf16 weight, or pk["w" + key + "_mx"] its MXFP8 codes + scales (quantised once, as
        _mx_quantize_linear does at load, model_fast.py:1384-1400); pk["b" + key] the bf16 bias."""
        if self._mx_name(key) in self.mx_linears:
            pk["w" + key + "_mx"] = kernels.mx_quantize(b(lin.weight), fmt=self.mx_fmt)[:2]
        else:
            pk["w" + key] = b(lin.weight)
        pk["b" + key] = b(lin.bias)

    def _linear_act(self, key, x, **kw):
        """One camera-FiLM MLP layer on the bf16 GEMM or, under lin_mx, on the MXFP8 GEMM."""
        pk = self._packed
        if "w" + key + "_mx" in pk:
            xq, xs, _ = kernels.mx_quantize(x, fmt=self.mx_fmt)
            return kernels.mx_linear_act(xq, xs, *pk["w" + key + "_mx"], pk["b" + key], fmt=self.mx_fmt, **kw)
        return kernels.linear_act(x, pk["w" + key], pk["b" + key], **kw)

    @torch.no_grad()
    def cam_film(self, c2ws_plucker_emb):
        """Camera FiLM parameters (cam_scale, cam_shift) of this block for the chunk's camera condition
        [1, L, C] (reference model_fast.py:2882-2891): silu(l1(c)) -> l2(.) + c -> (scale_layer, shift_layer),
        every Linear a tcgen05 GEMM. Depends only on the camera condition, so callers hoist it per chunk."""
        if self._packed is None:
            self.prepare()
        pk = self._packed
        if "bc1" not in pk:
            raise ValueError("cam_film needs prepare(with_cam=True)")
        C = self.dim
        c = c2ws_plucker_emb.reshape(-1, C).to(BF16).contiguous()
        h1 = self._linear_act("c1", c, silu=True)
        h2 = self._linear_act("c2", h1, addend=c)
        scale = self._linear_act("cs", h2)
        shift = self._linear_act("csh", h2)
        shape = c2ws_plucker_emb.shape[:-1] + (C,)
        return scale.view(shape), shift.view(shape)

    def workspace(self, rows, device):
        if self._ws is None or not self._ws.fits(rows, self.dim, self.ffn_dim, device):
            self._ws = Workspace(rows, self.dim, self.ffn_dim, device)
        return self._ws

    # ------------------------------------------------------------------ cross cache
    @torch.no_grad()
    def fill_cross_cache(self, context, crossattn_cache):
        """First call of a generation: K = RMSNorm(Wk ctx + bk), V = Wv ctx + bv into the cache
        (reference model_fast.py:2784-2798); with cross_dedup > 0 also the log-multiplicity bias."""
        pk = self._packed
        C = self.dim
        ctx = context.reshape(-1, C).to(BF16).contiguous()
        T = ctx.shape[0]
        kc = crossattn_cache["k"].view(T, C)
        vc = crossattn_cache["v"].view(T, C)
        k_raw = torch.empty(T, C, dtype=BF16, device=ctx.device)
        ss = torch.empty(T, dtype=torch.float32, device=ctx.device)
        fmt = self.mx_fmt
        cq = kernels.mx_quantize(ctx, fmt=fmt)[:2] if ("wck_mx" in pk or "wcv_mx" in pk) else None
        if "wck_mx" in pk:
            kernels.mx_linear_rowss(*cq, *pk["wck_mx"], pk["bck"], k_raw, ss, fmt=fmt)
        else:
            kernels.linear_rowss(ctx, pk["wck"], pk["bck"], k_raw, ss)
        kernels.rmsnorm_rope(k_raw, ss, pk["gck"], self.eps, kc)
        if "wcv_mx" in pk:
            kernels.mx_linear(*cq, *pk["wcv_mx"], pk["bcv"], out=vc, fmt=fmt)
        else:
            kernels.gemm_bf16(ctx, pk["wcv"], pk["bcv"], out=vc)
        if self.cross_dedup:
            crossattn_cache["mult"] = cross_dedup_bias(kc.view(T, self.num_heads, HEAD_DIM),
                                                       vc.view(T, self.num_heads, HEAD_DIM), self.cross_dedup)
        if "is_init" in crossattn_cache:
            crossattn_cache["is_init"].fill_(1)

    # ------------------------------------------------------------------ self-attention scheduling
    _comm_streams = {}

    def _self_attention(self, ws, k_chunks, v_chunks, L, chunk_rows, p):
        """Attention of the local queries over (leading..., destination).

        With sequence parallelism (p > 1) the destination chunk still has to be all-gathered. On CUDA the
        gather runs on copy engines from a side stream while ONE attention launch covers the whole window:
        its CTAs reach the destination chunk last and wait in-kernel for the copy engines' completion flag
        (the reference attends cached chunks while the gather is in flight the same way,
        model_fast.py:2033-2110). The windows (one head's pair of 128-row query tiles against every key) that
        the last full wave of CTAs leaves over are cut into key ranges, so that they fill the SMs that wave leaves
        idle, and merged (kernels.chunk_attention_tail)."""
        C, H = self.dim, self.num_heads
        rows = [k.numel() // C for k in k_chunks]
        k_dst, v_dst = k_chunks[-1], v_chunks[-1]
        tail_ws, pieces = ws.attn_tail(H, rows)
        pk = sp.peer_kv(k_dst.view(chunk_rows, C), L) if p > 1 else None
        if pk is None:
            if p > 1:
                sp.gather_kv_inplace(k_dst.view(chunk_rows, C), v_dst.view(chunk_rows, C), L)
            kernels.chunk_attention_tail(ws.q, k_chunks, v_chunks, tail_ws, out=ws.attn, pieces=pieces)
            return
        dev = ws.q.device
        comm = self._comm_streams.get(dev)
        if comm is None:
            comm = self._comm_streams[dev] = torch.cuda.Stream(device=dev)
        main = torch.cuda.current_stream(dev)
        k2d, v2d = k_dst.view(chunk_rows, C), v_dst.view(chunk_rows, C)
        pk.stage(k2d, v2d)                       # on this stream, so nothing of the exchange waits for an SM later
        ready = torch.cuda.Event()
        ready.record(main)
        with torch.cuda.stream(comm):
            comm.wait_event(ready)
            pk.finish(k2d, v2d)
        kernels.chunk_attention_tail(ws.q, k_chunks, v_chunks, tail_ws, out=ws.attn, pieces=pieces,
                                     gate_flag_ptr=pk.gathered_flag, gate_value=pk.epoch, gate_chunk=len(k_chunks) - 1)
        main.wait_stream(comm)                   # the destination chunk is complete for the caller

    # ------------------------------------------------------------------ forward
    def forward(self, x, e, seq_lens=None, grid_sizes=None, freqs=None, context=None, context_lens=None,
                dit_cond_dict=None, kv_cache=None, crossattn_cache=None, current_start=0,
                max_attention_size=1_000_000, frame_seqlen=None, cross_attn_first_call=None, seq_lens_int=None,
                sp_start_row=0, sp_rows=None, rope_grids=None, rope_local_grid=None, kv_write_start=None,
                kv_write_end=None, kv_roll_dst=0, kv_roll_src=0, kv_roll_len=0, kv_current_end=None,
                kv_chunks=None, grid_ints=None, fused=None, kv_write=True, kv_only=False):
        """x [1, L, C] fp32 (this rank's token shard under sequence parallelism), e [1, 1, 6, C] fp32
        -> new x (fp32). Writes the chunk's roped K and V into kv_chunks[0][-1] / kv_chunks[1][-1]; with
        kv_write=False (LINGBOT_STEP_NOWRITE: the denoise steps, model_fast.py:2135-2143, :3821-3835) the new
        chunk's K and V are attended from scratch and the destination slot is left unchanged."""
        if kv_chunks is None:
            raise ValueError("the B200 block serves the chunked KV cache: pass kv_chunks=(k_chunks, v_chunks)")
        if fused is not None or kv_roll_len:
            raise ValueError("fused commit/roll variants of the Trainium path are not part of the B200 block")
        if crossattn_cache is None or context is None:
            raise ValueError("pass the text context and its crossattn_cache dict")
        out = x.detach().float().reshape(-1, self.dim).clone()
        grid = self._grid(grid_ints, grid_sizes, rope_local_grid)
        if frame_seqlen is None:
            frame_seqlen = grid[1] * grid[2]
        start_frame = int(current_start) // int(frame_seqlen)
        if freqs is None:
            freqs = rope.rope_freqs()
        first = cross_attn_first_call
        if first is None:
            first = int(crossattn_cache["is_init"].reshape(-1)[0].item()) == 0
        film = None
        if dit_cond_dict is not None:
            if "cam_film" not in dit_cond_dict:
                raise ValueError("dit_cond_dict must carry the hoisted 'cam_film' (scale, shift)")
            film = dit_cond_dict["cam_film"]
        self.forward_inplace(out, e, kv_chunks[0], kv_chunks[1], context, crossattn_cache, grid, start_frame,
                             freqs, film=film, fill_cross=bool(first), kv_only=kv_only, kv_write=kv_write)
        return out.view(x.shape) if x.dtype == torch.float32 else out.view(x.shape).to(x.dtype)

    @staticmethod
    def _grid(grid_ints, grid_sizes, local_grid):
        if grid_ints is not None:
            g = grid_ints[0]
        elif local_grid is not None and not torch.is_tensor(local_grid):
            g = local_grid[0]
        elif grid_sizes is not None:
            g = grid_sizes[0].tolist() if torch.is_tensor(grid_sizes) else grid_sizes[0]
        else:
            raise ValueError("need the chunk's (frames, h, w) grid")
        return tuple(int(v) for v in g)

    def forward_inplace(self, xf, e, k_chunks, v_chunks, context, crossattn_cache, grid, start_frame, freqs,
                        film=None, fill_cross=False, kv_only=False, ws=None, attn_events=None, phases=None,
                        kv_write=True):
        """The block on the fp32 residual xf [L_local, C] (updated in place). attn_events: optional list
        that receives a (start, end) pair of CUDA events around the self-attention kernel. phases: optional
        list that receives (name, event) marks after each step, for per-phase timing. kv_write=False: the new
        chunk's K/V go to workspace scratch instead of the destination chunk, which is not modified."""
        mark = (lambda name: phases.append((name, _event()))) if phases is not None else (lambda name: None)
        mark("start")
        if self._packed is None:
            self.prepare()
        pk = self._packed
        C, H, eps = self.dim, self.num_heads, self.eps
        dev = xf.device
        L = xf.shape[0]
        ws = ws if ws is not None else self.workspace(L, dev)
        if fill_cross:
            self.fill_cross_cache(context, crossattn_cache)
        em = (pk["mod"] + e.reshape(6, C).float()).contiguous()
        k_dst, v_dst = k_chunks[-1], v_chunks[-1]
        chunk_rows = k_dst.numel() // C
        if not kv_write:
            if kv_only:
                raise ValueError("kv_only computes the cache entries: it needs kv_write=True")
            k_dst, v_dst = ws.new_kv(chunk_rows)
            k_chunks, v_chunks = list(k_chunks[:-1]) + [k_dst], list(v_chunks[:-1]) + [v_dst]
        p = sp.world() if sp.active() else 1
        if chunk_rows != L * p:
            raise ValueError(f"destination chunk holds {chunk_rows} tokens, expected {L} x {p} ranks")
        row0 = (sp.rank() * L) if p > 1 else 0
        f, gh, gw = grid
        if f * gh * gw != chunk_rows:
            raise ValueError(f"grid {grid} does not match the chunk's {chunk_rows} tokens")
        cos, sin = rope.rope_tables(freqs, grid, start_frame, dev)
        rp = (cos, sin, f)
        ss_q, ss_k = ws.ss_q, ws.ss_k

        # self-attention
        fmt = self.mx_fmt
        if "wqkv_mx" in pk:
            kernels.layernorm_mod_mx(xf, eps, em[1], em[0], ws.hq, ws.hs, fmt=fmt)
            mark("ln1")
            kernels.mx_qkv_proj(ws.hq, ws.hs, *pk["wqkv_mx"], pk["bqkv"], ws.q_raw, ws.k_raw, ss_q, ss_k, v_dst,
                                v_row_off=row0, fmt=fmt)
        else:
            kernels.layernorm_mod(xf, eps, ws.h, scale=em[1], shift=em[0])
            mark("ln1")
            kernels.qkv_proj(ws.h, pk["wqkv"], pk["bqkv"], ws.q_raw, ws.k_raw, ss_q, ss_k, v_dst, v_row_off=row0)
        mark("qkv")
        kernels.qk_rmsnorm_rope(ws.q_raw, ss_q, pk["gq"], ws.q, ws.k_raw, ss_k, pk["gk"], k_dst, eps, rp, grid,
                                tok0=row0, k_row_off=row0, rope_bf16=rope.ROPE_DTYPE == torch.bfloat16)
        mark("qk_norm_rope")
        if kv_only:
            if p > 1:
                sp.gather_kv_inplace(k_dst.view(chunk_rows, C), v_dst.view(chunk_rows, C), L)
            return xf
        if attn_events is not None:
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
        self._self_attention(ws, list(k_chunks), list(v_chunks), L, chunk_rows, p)
        if attn_events is not None:
            ev1.record()
            attn_events.append((ev0, ev1))
        mark("self_attn")
        fs, ft = (film[0].reshape(-1, C), film[1].reshape(-1, C)) if film is not None else (None, None)
        if fs is not None:
            fs, ft = fs.to(BF16).contiguous(), ft.to(BF16).contiguous()
        if "wo_mx" in pk:
            kernels.mx_quantize(ws.attn, data=ws.hq, scales=ws.hs, fmt=fmt)
            kernels.mx_linear_residual(ws.hq, ws.hs, *pk["wo_mx"], pk["bo"], xf, gate=em[2], film_scale=fs, fmt=fmt,
                                       film_shift=ft)
        else:
            kernels.linear_residual(ws.attn, pk["wo"], pk["bo"], xf, gate=em[2], film_scale=fs, film_shift=ft)
        mark("o_proj_film")

        # cross-attention
        if not self.cross_attn_norm:
            raise ValueError("cross_attn_norm=False is not supported by the B200 block")
        if "wcq_mx" in pk:
            kernels.layernorm_affine_mx(xf, eps, pk["n3w"], pk["n3b"], ws.hq, ws.hs, fmt=fmt)
            mark("ln3")
            kernels.mx_linear_rowss(ws.hq, ws.hs, *pk["wcq_mx"], pk["bcq"], ws.q_raw, ss_q, fmt=fmt)
        else:
            kernels.layernorm_mod(xf, eps, ws.h, weight=pk["n3w"], bias=pk["n3b"])
            mark("ln3")
            kernels.linear_rowss(ws.h, pk["wcq"], pk["bcq"], ws.q_raw, ss_q)
        kernels.rmsnorm_rope(ws.q_raw, ss_q, pk["gcq"], eps, ws.q)
        mark("cross_q")
        T = crossattn_cache["k"].numel() // C
        kc, vc = crossattn_cache["k"].view(T, C), crossattn_cache["v"].view(T, C)
        bias = None
        if self.cross_dedup:
            n = self.cross_dedup
            kc, vc, bias = kc[:n], vc[:n], crossattn_cache["mult"]
        kernels.chunk_attention(ws.q, [kc], [vc], key_bias=bias, out=ws.attn)
        mark("cross_attn")
        if "wco_mx" in pk:
            kernels.mx_quantize(ws.attn, data=ws.hq, scales=ws.hs, fmt=fmt)
            kernels.mx_linear_residual(ws.hq, ws.hs, *pk["wco_mx"], pk["bco"], xf, fmt=fmt)
        else:
            kernels.linear_residual(ws.attn, pk["wco"], pk["bco"], xf)
        mark("cross_o")

        # FFN
        if self.ffn_mx and self.mx_pipe == "mxf8":
            kernels.layernorm_mod_mx(xf, eps, em[4], em[3], ws.hq, ws.hs, fmt=fmt)
            mark("ln2")
            kernels.mx_linear_gelu(ws.hq, ws.hs, *pk["w1_mx"], pk["b1"], ws.uq, ws.us, fmt=fmt)
            mark("ffn_up")
            kernels.mx_linear_residual(ws.uq, ws.us, *pk["w2_mx"], pk["b2"], xf, gate=em[5], fmt=fmt)
        else:
            kernels.layernorm_mod(xf, eps, ws.h, scale=em[4], shift=em[3], mx_qdq=self.ffn_mx)
            kernels.linear_gelu(ws.h, pk["w1"], pk["b1"], ws.u, mx_qdq=self.ffn_mx)
            kernels.linear_residual(ws.u, pk["w2"], pk["b2"], xf, gate=em[5])
        mark("ffn_down")
        return xf


KERNELS_PER_BLOCK = 13  # plus the merge of the self-attention's cut windows when its tail schedule cuts some
