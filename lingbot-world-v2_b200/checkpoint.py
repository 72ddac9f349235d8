"""Loading a causal-fast DiT checkpoint into CausalWanModel.

Mirrors the reference loader (wan/image2video.py:306-400): the DiT folder is `checkpoint_dir/<subfolder>`
when it exists (the 14B causal-fast upload keeps its weights under `transformers/`), else the root; weights
are a sharded safetensors dump with a `*.safetensors.index.json` weight map, or one `model.safetensors` /
`diffusion_pytorch_model.safetensors`; the architecture comes from `config.json` when present, else from
the task config (`_dit_kwargs_from_config`). Parameter names are the reference's (`blocks.{i}.self_attn.q.weight`,
`head.modulation`, ...), so the state dict loads unchanged.

Dtypes follow the reference pipeline (`model.to(torch_dtype)` at load, the timestep MLPs, the head and each
block's modulation / norm3 evaluated in fp32 under its fp32 autocast): bf16 parameters except those, which
are kept fp32.
"""
import json
import os

import torch

from .model import CausalWanModel

_INDEX_NAMES = ("model.safetensors.index.json", "diffusion_pytorch_model.safetensors.index.json")
_SINGLE_NAMES = ("model.safetensors", "diffusion_pytorch_model.safetensors")
_CONFIG_KEYS = ("model_type", "patch_size", "text_len", "in_dim", "dim", "ffn_dim", "freq_dim", "text_dim",
                "out_dim", "num_heads", "num_layers", "qk_norm", "cross_attn_norm", "eps")


def resolve_dit_dir(checkpoint_dir, subfolder="transformers"):
    """checkpoint_dir/subfolder when it is a directory, else checkpoint_dir (image2video.py:306-316)."""
    if subfolder:
        cand = os.path.join(checkpoint_dir, subfolder)
        if os.path.isdir(cand):
            return cand
    return checkpoint_dir


def load_state_dict(dit_dir, device="cpu"):
    """The (possibly sharded) safetensors state dict of a DiT folder (image2video.py:319-348)."""
    from safetensors.torch import load_file
    for name in _INDEX_NAMES:
        path = os.path.join(dit_dir, name)
        if os.path.isfile(path):
            with open(path) as f:
                index = json.load(f)
            state = {}
            for shard in sorted(set(index["weight_map"].values())):
                state.update(load_file(os.path.join(dit_dir, shard), device=str(device)))
            missing = set(index["weight_map"]) - set(state)
            if missing:
                raise ValueError(f"{dit_dir}: the index lists tensors no shard holds: {sorted(missing)[:5]}")
            return state
    for name in _SINGLE_NAMES:
        path = os.path.join(dit_dir, name)
        if os.path.isfile(path):
            return load_file(path, device=str(device))
    raise FileNotFoundError(f"no safetensors weights (index or single file) in {dit_dir}")


def model_kwargs(dit_dir, config=None, **overrides):
    """Architecture arguments: config.json in the DiT folder, else the task config object (attributes named
    as in wan/configs, image2video.py:351-370), then `overrides`."""
    kw = {}
    path = os.path.join(dit_dir, "config.json")
    if os.path.isfile(path):
        with open(path) as f:
            cfg = json.load(f)
        kw = {k: cfg[k] for k in _CONFIG_KEYS if k in cfg}
    elif config is not None:
        kw = dict(model_type="i2v", patch_size=tuple(config.patch_size), text_len=config.text_len,
                  in_dim=getattr(config, "in_dim", 36), dim=config.dim, ffn_dim=config.ffn_dim,
                  freq_dim=config.freq_dim, text_dim=getattr(config, "text_dim", 4096),
                  out_dim=getattr(config, "out_dim", 16), num_heads=config.num_heads, num_layers=config.num_layers,
                  qk_norm=config.qk_norm, cross_attn_norm=config.cross_attn_norm, eps=config.eps)
    else:
        raise ValueError(f"{dit_dir} has no config.json: pass the task config")
    if "patch_size" in kw:
        kw["patch_size"] = tuple(kw["patch_size"])
    kw.update(overrides)
    return kw


def _fp32_names(model):
    names = set()
    for pre in ("time_embedding", "time_projection", "head"):
        names |= {f"{pre}.{n}" for n, _ in getattr(model, pre).named_parameters()}
    for i, blk in enumerate(model.blocks):
        names.add(f"blocks.{i}.modulation")
        names |= {f"blocks.{i}.norm3.{n}" for n, _ in blk.norm3.named_parameters()}
    return names


@torch.no_grad()
def load_model(checkpoint_dir, subfolder="transformers", config=None, device="cuda", ffn_mx=False, cross_dedup=0,
               strict=True, pack=True, lin_mx=False, lin_mx_skip=(), **overrides):
    """CausalWanModel with the checkpoint's weights on `device`, packed for the kernels. The model is built on
    the meta device and materialised once in its final dtypes (no fp32 copy of the bf16 weights). ffn_mx /
    lin_mx / lin_mx_skip: LINGBOT_FFN_MX / LINGBOT_LIN_MX / LINGBOT_LIN_MX_SKIP (weights quantised at prepare). strict:
    every model parameter must come from the checkpoint (the reference only warns about missing keys);
    unexpected checkpoint keys are reported in the returned list either way. pack=False skips the kernel
    packing (prepare(), CUDA only)."""
    dit_dir = resolve_dit_dir(checkpoint_dir, subfolder)
    kw = model_kwargs(dit_dir, config, ffn_mx=ffn_mx, cross_dedup=cross_dedup, lin_mx=lin_mx,
                      lin_mx_skip=tuple(lin_mx_skip), **overrides)
    with torch.device("meta"):
        model = CausalWanModel(**kw)
    fp32 = _fp32_names(model)
    state = load_state_dict(dit_dir)
    params = dict(model.named_parameters())
    missing = [n for n in params if n not in state]
    unexpected = [n for n in state if n not in params]
    if strict and missing:
        raise ValueError(f"checkpoint {dit_dir} lacks {len(missing)} parameters, e.g. {missing[:5]}")
    for n, p in params.items():
        if n in state and tuple(state[n].shape) != tuple(p.shape):
            raise ValueError(f"{n}: checkpoint shape {tuple(state[n].shape)} vs model {tuple(p.shape)}")
    model = model.to_empty(device=device)
    for n, p in model.named_parameters():
        dtype = torch.float32 if n in fp32 else torch.bfloat16
        p.data = (state[n] if n in state else torch.zeros(p.shape)).to(device=device, dtype=dtype)
    if pack:
        model.prepare()
    return model, unexpected
