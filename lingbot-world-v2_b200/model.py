"""The block loop of one denoising step: N CausalWanAttentionBlocks over one query chunk.

The reference runs `for block in self.blocks: x = block(x, kv_chunks=(ks, vs), ...)` inside
WanModelFast.forward (wan/modules/model_fast.py:3830-3852) with per-block chunk lists from
ordered_chunks_by_block (chunked_kv_cache.py:179-182). BlockStack does the same on one fp32
residual buffer updated in place, with one shared scratch workspace for all blocks.
"""
import torch
import torch.nn as nn

from .block import CausalWanAttentionBlock, Workspace

CONFIGS = {
    # wan/configs/wan_i2v_1_3B.py:21-33 and wan_i2v_A14B.py:16-33 (text_len 512, shared_config.py:9-12)
    "1.3B": dict(dim=1536, ffn_dim=8960, num_heads=12, num_layers=30),
    "14B": dict(dim=5120, ffn_dim=13824, num_heads=40, num_layers=40),
}


class BlockStack(nn.Module):
    def __init__(self, num_layers, dim, ffn_dim, num_heads, eps=1e-6, ffn_mx=True, cross_dedup=0):
        super().__init__()
        self.dim, self.ffn_dim, self.num_heads = dim, ffn_dim, num_heads
        self.blocks = nn.ModuleList([
            CausalWanAttentionBlock(dim, ffn_dim, num_heads, qk_norm=True, cross_attn_norm=True, eps=eps,
                                    ffn_mx=ffn_mx, cross_dedup=cross_dedup) for _ in range(num_layers)])
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
    def synthetic(cls, num_layers, dim, ffn_dim, num_heads, device, seed=0, ffn_mx=True, peaked=False):
        """Build on the meta device, materialise bf16 weights on `device`, fill with the benchmark
        distributions and pack them for the kernels (source copies freed)."""
        with torch.device("meta"):
            st = cls(num_layers, dim, ffn_dim, num_heads, ffn_mx=ffn_mx)
        st = st.to(torch.bfloat16).to_empty(device=device)
        for blk in st.blocks:
            blk.modulation.data = blk.modulation.data.float()
            blk.norm3.weight.data = blk.norm3.weight.data.float()
            blk.norm3.bias.data = blk.norm3.bias.data.float()
        g = torch.Generator(device=device).manual_seed(seed)
        init_synthetic_(st, g, peaked=peaked)
        for blk in st.blocks:
            blk.prepare(free_sources=True, with_cam=False)   # the benchmark feeds hoisted FiLM tensors
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
