"""The block loop of one denoising step (BlockStack) and the whole causal-fast model around it (CausalWanModel).

The reference runs `for block in self.blocks: x = block(x, kv_chunks=(ks, vs), ...)` inside
WanModelFast.forward (wan/modules/model_fast.py:3830-3852) with per-block chunk lists from
ordered_chunks_by_block (chunked_kv_cache.py:179-182). BlockStack does the same on one fp32
residual buffer updated in place, with one shared scratch workspace for all blocks.
"""
import math

import torch
import torch.nn as nn

from . import kernels, rope, sp
from .block import CausalWanAttentionBlock, Workspace

CONFIGS = {
    # wan/configs/wan_i2v_1_3B.py:21-33 and wan_i2v_A14B.py:16-33 (text_len 512, shared_config.py:9-12)
    "1.3B": dict(dim=1536, ffn_dim=8960, num_heads=12, num_layers=30),
    "14B": dict(dim=5120, ffn_dim=13824, num_heads=40, num_layers=40),
}


class BlockStack(nn.Module):
    def __init__(self, num_layers, dim, ffn_dim, num_heads, eps=1e-6, ffn_mx=True, cross_dedup=0, lin_mx=False,
                 lin_mx_skip=()):
        super().__init__()
        self.dim, self.ffn_dim, self.num_heads = dim, ffn_dim, num_heads
        self.blocks = nn.ModuleList([
            CausalWanAttentionBlock(dim, ffn_dim, num_heads, qk_norm=True, cross_attn_norm=True, eps=eps,
                                    ffn_mx=ffn_mx, cross_dedup=cross_dedup, lin_mx=lin_mx, lin_mx_skip=lin_mx_skip)
            for _ in range(num_layers)])
        self._ws = None

    def prepare(self):
        for b in self.blocks:
            b.prepare()

    def forward_chunk(self, xf, e, kv_chunks_by_block, context, cross_caches, grid, start_frame, freqs, films=None,
                      fill_cross=False, attn_events=None, phases=None):
        """xf [L_local, C] fp32 residual (updated in place); kv_chunks_by_block = (ks, vs) with ks[i] the
        ordered K chunk list of block i; films[i] = (scale, shift) or None."""
        L = xf.shape[0]
        if self._ws is None or not self._ws.fits(L, self.dim, self.ffn_dim, xf.device):
            self._ws = Workspace(L, self.dim, self.ffn_dim, xf.device)
        ks, vs = kv_chunks_by_block
        for i, blk in enumerate(self.blocks):
            blk.forward_inplace(xf, e, ks[i], vs[i], context, cross_caches[i], grid, start_frame, freqs,
                                film=None if films is None else films[i], fill_cross=fill_cross, ws=self._ws,
                                attn_events=attn_events, phases=phases)
        return xf

    @classmethod
    def synthetic(cls, num_layers, dim, ffn_dim, num_heads, device, seed=0, ffn_mx=True, peaked=False, lin_mx=False,
                  free_sources=True):
        """Build on the meta device, materialise bf16 weights on `device`, fill with the benchmark
        distributions and pack them for the kernels (source copies freed unless free_sources=False). The
        generator draws block by block, so the first blocks of two stacks built with the same seed are equal."""
        with torch.device("meta"):
            st = cls(num_layers, dim, ffn_dim, num_heads, ffn_mx=ffn_mx, lin_mx=lin_mx)
        st = st.to(torch.bfloat16).to_empty(device=device)
        for blk in st.blocks:
            blk.modulation.data = blk.modulation.data.float()
            blk.norm3.weight.data = blk.norm3.weight.data.float()
            blk.norm3.bias.data = blk.norm3.bias.data.float()
        g = torch.Generator(device=device).manual_seed(seed)
        init_synthetic_(st, g, peaked=peaked)
        for blk in st.blocks:
            blk.prepare(free_sources=free_sources, with_cam=False)   # the benchmark feeds hoisted FiLM tensors
        return st


@torch.no_grad()
def init_synthetic_(stack, generator, peaked=False):
    """Benchmark initialisation: Linear weights/biases ~N(0, 0.02); RMSNorm gammas and the norm3 affine
    ~N(0, 0.02) (or 1 + N(0, 0.02) when peaked); modulation ~N(0, 0.1)."""
    for blk in stack.blocks:
        for name, prm in blk.named_parameters():
            if name.startswith("cam_"):
                continue
            if name == "modulation":
                prm.copy_(torch.randn(prm.shape, generator=generator, device=prm.device) * 0.1)
            elif ("norm_q" in name or "norm_k" in name or name.startswith("norm3.weight")) and peaked:
                prm.copy_(1.0 + torch.randn(prm.shape, generator=generator, device=prm.device) * 0.02)
            else:
                prm.copy_(torch.randn(prm.shape, generator=generator, device=prm.device) * 0.02)
    return stack


class CausalHead(nn.Module):
    """CausalHead (wan/modules/model_fast.py:3119-3148): LN(x) * (1 + e1) + e0, e = modulation + e, then a Linear
    to out_dim * prod(patch) per token (here LayerNorm kernel + tcgen05 GEMM)."""

    def __init__(self, dim, out_dim, patch_size, eps=1e-6):
        super().__init__()
        self.dim, self.out_dim, self.patch_size, self.eps = dim, out_dim, patch_size, eps
        self.norm = nn.Identity()        # WanLayerNorm without affine: no parameters
        self.head = nn.Linear(dim, math.prod(patch_size) * out_dim)
        self.modulation = nn.Parameter(torch.randn(1, 2, dim) / dim ** 0.5)

    def forward(self, x, e):
        """x [L, dim] fp32, e [dim] fp32 -> [L, out_dim * prod(patch)] fp32."""
        m = (self.modulation.detach().float().reshape(2, self.dim) + e.float().reshape(1, self.dim)).contiguous()
        h = torch.empty(x.shape[0], self.dim, dtype=torch.bfloat16, device=x.device)
        kernels.layernorm_mod(x.contiguous(), self.eps, h, scale=m[1], shift=m[0])
        w = self.head.weight.detach().to(torch.bfloat16).contiguous()
        b = self.head.bias.detach().to(torch.bfloat16).contiguous()
        return kernels.gemm_bf16(h, w, b).float()


def patch_tokens(v, patch):
    """[C, F, H, W] -> [F/pt * H/ph * W/pw, C * pt * ph * pw] (frame-major tokens; columns in Conv3d weight order)."""
    c, f, h, w = v.shape
    pt, ph, pw = patch
    t = v.reshape(c, f // pt, pt, h // ph, ph, w // pw, pw)
    return t.permute(1, 3, 5, 0, 2, 4, 6).reshape((f // pt) * (h // ph) * (w // pw), c * pt * ph * pw)


def sinusoidal_embedding_1d(dim, position):
    """wan/modules/model.py:16-26: cos | sin of position * 10000^(-i/half), in fp64."""
    half = dim // 2
    position = position.to(torch.float64)
    s = torch.outer(position, torch.pow(10000, -torch.arange(half, device=position.device).to(position).div(half)))
    return torch.cat([torch.cos(s), torch.sin(s)], dim=1)


class CausalWanModel(nn.Module):
    """WanModelFast (wan/modules/model_fast.py:3151-3283) around the B200 blocks, with the reference's module
    names and state-dict keys, on its default causal-fast path (forward :3283-3935): chunked KV cache routed by
    chunk_routing, hoisted camera FiLM, exact attention, flat sequence parallelism.

    Every token-wise Linear (patch embedding as a GEMM over 1x2x2 patches, the camera embedding and its MLP,
    the text embedding, the head) runs on the library's tcgen05 GEMMs; the timestep MLP (one row per
    forward, fp32 in the reference) is a plain fp32 matmul, cached per timestep value like the reference's."""

    def __init__(self, model_type="i2v", patch_size=(1, 2, 2), text_len=512, in_dim=16, dim=2048, ffn_dim=8192,
                 freq_dim=256, text_dim=4096, out_dim=16, num_heads=16, num_layers=32, local_attn_size=-1,
                 sink_size=0, qk_norm=True, cross_attn_norm=True, eps=1e-6, ffn_mx=False, cross_dedup=0,
                 lin_mx=False, lin_mx_skip=()):
        super().__init__()
        if model_type not in ("t2v", "i2v"):
            raise ValueError("model_type is 't2v' or 'i2v'")
        if tuple(patch_size) != (1, 2, 2):
            raise ValueError("the B200 model serves patch_size (1, 2, 2)")
        self.model_type, self.patch_size, self.text_len = model_type, tuple(patch_size), text_len
        self.in_dim, self.dim, self.ffn_dim, self.freq_dim = in_dim, dim, ffn_dim, freq_dim
        self.text_dim, self.out_dim, self.num_heads, self.num_layers, self.eps = text_dim, out_dim, num_heads, num_layers, eps
        control_dim = 6
        self.patch_embedding = nn.Conv3d(in_dim, dim, kernel_size=patch_size, stride=patch_size)
        self.patch_embedding_wancamctrl = nn.Linear(control_dim * 64 * math.prod(patch_size), dim)
        self.c2ws_hidden_states_layer1 = nn.Linear(dim, dim)
        self.c2ws_hidden_states_layer2 = nn.Linear(dim, dim)
        self.text_embedding = nn.Sequential(nn.Linear(text_dim, dim), nn.GELU(approximate="tanh"), nn.Linear(dim, dim))
        self.time_embedding = nn.Sequential(nn.Linear(freq_dim, dim), nn.SiLU(), nn.Linear(dim, dim))
        self.time_projection = nn.Sequential(nn.SiLU(), nn.Linear(dim, dim * 6))
        self.blocks = nn.ModuleList([
            CausalWanAttentionBlock(dim, ffn_dim, num_heads, local_attn_size, sink_size, qk_norm, cross_attn_norm, eps,
                                    ffn_mx=ffn_mx, cross_dedup=cross_dedup, lin_mx=lin_mx, lin_mx_skip=lin_mx_skip)
            for _ in range(num_layers)])
        self.head = CausalHead(dim, out_dim, patch_size, eps)
        self.freqs = None
        self._packed = None
        self._t_cache = {}
        self._ctx_cache = None

    @torch.no_grad()
    def prepare(self):
        """Pack the embedding weights for the kernels (bf16, K padded to a multiple of 64) and the blocks."""
        b = lambda t: t.detach().to(torch.bfloat16).contiguous()  # noqa: E731
        w = self.patch_embedding.weight.detach().reshape(self.dim, -1)
        k = w.shape[1]
        kp = (k + 63) // 64 * 64
        pk = {"patch_w": b(torch.nn.functional.pad(w, (0, kp - k))), "patch_b": b(self.patch_embedding.bias),
              "patch_k": k, "patch_kp": kp}
        pk["cam_w"], pk["cam_b"] = b(self.patch_embedding_wancamctrl.weight), b(self.patch_embedding_wancamctrl.bias)
        pk["c1_w"], pk["c1_b"] = b(self.c2ws_hidden_states_layer1.weight), b(self.c2ws_hidden_states_layer1.bias)
        pk["c2_w"], pk["c2_b"] = b(self.c2ws_hidden_states_layer2.weight), b(self.c2ws_hidden_states_layer2.bias)
        pk["t0_w"], pk["t0_b"] = b(self.text_embedding[0].weight), b(self.text_embedding[0].bias)
        pk["t2_w"], pk["t2_b"] = b(self.text_embedding[2].weight), b(self.text_embedding[2].bias)
        self._packed = pk
        for blk in self.blocks:
            blk.prepare(with_cam=True)
        self._t_cache, self._ctx_cache = {}, None
        return pk

    # ---------------------------------------------------------------- embeddings
    def _time(self, t):
        """e [dim], e0 [6, dim] (fp32) for one timestep value, cached per value (the reference caches by the
        host-side timestep key, model_fast.py:3425-3446)."""
        key = (float(t.reshape(-1)[0]), str(t.device))
        hit = self._t_cache.get(key)
        if hit is None:
            F_ = torch.nn.functional
            s = sinusoidal_embedding_1d(self.freq_dim, t.reshape(-1)[:1]).float()
            te, tp = self.time_embedding, self.time_projection
            e = F_.linear(s, te[0].weight.float(), te[0].bias.float())
            e = F_.linear(F_.silu(e), te[2].weight.float(), te[2].bias.float())
            e0 = F_.linear(F_.silu(e), tp[1].weight.float(), tp[1].bias.float())
            hit = self._t_cache[key] = (e.reshape(self.dim).contiguous(), e0.reshape(1, 1, 6, self.dim).contiguous())
        return hit

    def _text(self, ctx):
        if self._ctx_cache is not None and self._ctx_cache[0] is ctx:
            return self._ctx_cache[1]
        pk = self._packed
        c = torch.cat([ctx, ctx.new_zeros(self.text_len - ctx.shape[0], ctx.shape[1])]).to(torch.bfloat16).contiguous()
        h = torch.empty(self.text_len, self.dim, dtype=torch.bfloat16, device=c.device)
        kernels.linear_gelu(c, pk["t0_w"], pk["t0_b"], h, mx_qdq=False)
        out = kernels.gemm_bf16(h, pk["t2_w"], pk["t2_b"])
        self._ctx_cache = (ctx, out)
        return out

    def _patch(self, x_cat):
        pk = self._packed
        a = patch_tokens(x_cat.to(torch.bfloat16), self.patch_size)
        a = torch.nn.functional.pad(a, (0, pk["patch_kp"] - pk["patch_k"])).contiguous()
        return kernels.gemm_bf16(a, pk["patch_w"], pk["patch_b"])

    def _camera(self, cam):
        """cam [1, 6*64, F, H, W] -> emb + layer2(silu(layer1(emb))) [L, dim] bf16 (model_fast.py:3505-3552)."""
        pk = self._packed
        c = patch_tokens(cam[0].to(torch.bfloat16), self.patch_size).contiguous()
        emb = kernels.gemm_bf16(c, pk["cam_w"], pk["cam_b"])
        h = kernels.linear_act(emb, pk["c1_w"], pk["c1_b"], silu=True)
        return kernels.linear_act(h, pk["c2_w"], pk["c2_b"], addend=emb)

    def unpatchify(self, u, grid):
        """[L, out_dim * 4] -> [out_dim, F, H, W] (model_fast.py:4419-4440)."""
        f, h, w = grid
        u = u[: f * h * w].reshape(f, h, w, *self.patch_size, self.out_dim)
        u = torch.einsum("fhwpqrc->cfphqwr", u)
        return u.reshape(self.out_dim, *[a * b for a, b in zip(grid, self.patch_size)])

    # ---------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, x, t, context, seq_len, y=None, dit_cond_dict=None, kv_cache=None, crossattn_cache=None,
                current_start=0, max_attention_size=1_000_000, frame_seqlen=None, cross_attn_first_call=None,
                skip_head=False, kv_commit=None):
        """x: [latent [C, F, H, W]] (one chunk), t: timestep [1], context: [prompt [rows, text_dim]], y: [condition]
        for i2v, dit_cond_dict={"c2ws_plucker_emb": [[1, 384, F, H, W]]} (optional), kv_cache: per block
        {"k": [chunks], "v": [chunks]} (allocate_self_kv_chunks), crossattn_cache: per block dict.
        Returns [out [out_dim, F, H, W] fp32], or None with skip_head (the KV-commit forward)."""
        from . import chunked_kv_cache as ckv
        if self._packed is None:
            self.prepare()
        if len(x) != 1 or len(context) != 1:
            raise ValueError("the B200 model runs one chunk per forward (len(x) == len(context) == 1)")
        if not kv_cache or not isinstance(kv_cache[0].get("k"), (list, tuple)):
            raise ValueError("the B200 model serves the chunked KV cache (allocate_self_kv_chunks)")
        if self.model_type == "i2v" and y is None:
            raise ValueError("i2v needs the conditioning y")
        rope.set_bf16_rope_for_forward(seq_len)   # the reference's switch to bf16 RoPE (model_fast.py:3348)
        u = torch.cat([x[0], y[0]], dim=0) if y is not None else x[0]
        grid = tuple(int(v) // p for v, p in zip(u.shape[1:], self.patch_size))
        L = grid[0] * grid[1] * grid[2]
        if L > seq_len:
            raise ValueError(f"{L} tokens exceed seq_len {seq_len}")
        dev = u.device
        tokens = self._patch(u).float()
        ctx = self._text(context[0])
        e, e0 = self._time(t.to(dev))
        films = None
        if dit_cond_dict is not None and "c2ws_plucker_emb" in dit_cond_dict:
            cam = self._camera(dit_cond_dict["c2ws_plucker_emb"][0])
            films = [blk.cam_film(cam) for blk in self.blocks]
        if sp.active():
            tokens = sp.shard_tokens(tokens)
            if films is not None:
                films = [(sp.shard_tokens(s), sp.shard_tokens(h)) for s, h in films]
        fs = int(frame_seqlen) if frame_seqlen is not None else grid[1] * grid[2]
        n_chunks = len(kv_cache[0]["k"])
        dest, leading = ckv.chunk_routing(int(current_start) // max(1, fs * grid[0]), n_chunks)
        ks, vs = ckv.ordered_chunks_by_block(kv_cache, dest, leading)
        if self.freqs is None:
            self.freqs = rope.rope_freqs()
        xf = tokens.reshape(1, -1, self.dim)
        for i, blk in enumerate(self.blocks):
            cond = {"cam_film": films[i]} if films is not None else None
            xf = blk(xf, e0, grid_ints=[grid], freqs=self.freqs, context=ctx.unsqueeze(0), dit_cond_dict=cond,
                     crossattn_cache=crossattn_cache[i], current_start=int(current_start), frame_seqlen=fs,
                     cross_attn_first_call=cross_attn_first_call, kv_chunks=(list(ks[i]), list(vs[i])))
        if skip_head:
            return None
        out = self.head(xf.reshape(-1, self.dim), e)
        if sp.active():
            out = sp.gather_tokens(out)
        return [self.unpatchify(out, grid)]

    @torch.no_grad()
    def forward_fused(self, xa, ya, cam_a, ta, ta_key, chunk_a, xb, yb, cam_b, tb, tb_key, chunk_b, context, seq_len,
                      kv_cache, crossattn_cache, frame_seqlen, max_attention_size=1_000_000):
        """Chunk a's KV-cache commit (clean latent xa at ta = 0) and chunk b's first denoise step (xb at tb), the
        reference's LINGBOT_FUSE_COMMIT forward (model_fast.py:3985-4097, called from image2video.py:1638-1649),
        with its signature and result ([b's output]). The reference packs both chunks into one forward so that a
        Trainium graph pays its per-block fixed costs once; here the two forwards run back to back on the stream
        (every GEMM of a 10,800-token chunk is already compute-bound, and the key sets are the same: a attends to
        its window before b's K/V overwrite the chunk b evicts, b to the shared chunks, fresh a and itself).
        ta_key / tb_key (host-side timestep cache keys) are not needed: timestep embeddings are cached by value.
        cam_a / cam_b: the c2ws_plucker_emb lists of the two chunks (or None)."""
        def start(x, chunk):
            return int(chunk) * (int(x.shape[1]) // self.patch_size[0]) * int(frame_seqlen)

        def cond(cam):
            return {"c2ws_plucker_emb": cam} if cam is not None else None
        self.forward([xa], ta, context, seq_len, y=[ya] if ya is not None else None, dit_cond_dict=cond(cam_a),
                     kv_cache=kv_cache, crossattn_cache=crossattn_cache, current_start=start(xa, chunk_a),
                     max_attention_size=max_attention_size, frame_seqlen=frame_seqlen, cross_attn_first_call=False,
                     skip_head=True)
        return self.forward([xb], tb, context, seq_len, y=[yb] if yb is not None else None, dit_cond_dict=cond(cam_b),
                            kv_cache=kv_cache, crossattn_cache=crossattn_cache, current_start=start(xb, chunk_b),
                            max_attention_size=max_attention_size, frame_seqlen=frame_seqlen,
                            cross_attn_first_call=False)
