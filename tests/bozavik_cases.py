"""Small Bozavik configurations and model folders with random weights, for the tests."""

from __future__ import annotations

import json
import os

import torch
from safetensors.torch import save_file

from tt_transformers_b200.weights import random_tensors


def mixer(kind, heads, dim, vdim, q_rank, kv_rank, rot_dim=0, rot_dims=None, base=10000.0):
    m = {"heads": heads, "dim": dim, "vdim": vdim, "q_rank": q_rank, "kv_rank": kv_rank, "scale": (dim + rot_dim) ** -0.5}
    if kind == "latent_attention_2":
        m.update(rot_dim=rot_dim, rot={"base": base, "dims": rot_dims or rot_dim})
    return m


def mlp(experts, top, ff, limit, shared_ff=None, shared_limit=None):
    out = {"kind": "moe", "router": {"experts": experts, "top": top}, "expert": {"ff": ff, "limit": limit}}
    if shared_ff:
        out["shared"] = {"ff": shared_ff, "limit": shared_limit}
    return out


def layer(kind, mixer_cfg, mlp_cfg):
    return {"type": kind, "mixer": mixer_cfg, "mlp": mlp_cfg}


def config(width, vocab, layers, residual_mult=0.7, eps=1e-5, embed_scale=2.0):
    return {"architecture": "Bozavik", "vocab": vocab, "width": width, "residual_mult": residual_mult,
            "norm": {"eps": eps}, "embedding": {"scale": embed_scale}, "layers": layers}


# sizes that the tensor-core kernels take (multiples of 16), both mixers, shared and unshared feed-forwards
ALIGNED = config(128, 300, [
    layer("latent_attention_2", mixer("latent_attention_2", 4, 32, 16, 48, 64, rot_dim=16, base=1000.0), mlp(6, 2, 48, 1.5, 64, 0.8)),
    layer("latent_attention", mixer("latent_attention", 3, 16, 32, 64, 48), mlp(4, 3, 32, 2.5)),
    layer("latent_attention", mixer("latent_attention", 8, 16, 16, 32, 32), None),
    layer("latent_attention_2", mixer("latent_attention_2", 2, 48, 32, 64, 80, rot_dim=32, rot_dims=16), mlp(5, 5, 64, 1.0, 32, 2.0)),
])

# sizes that only the general kernels take: odd widths and ranks, one head, one expert, top equal to 1
ODD = config(60, 131, [
    layer("latent_attention", mixer("latent_attention", 1, 12, 20, 28, 36), mlp(1, 1, 20, 3.0, 12, 1.0)),
    layer("latent_attention_2", mixer("latent_attention_2", 5, 6, 10, 18, 22, rot_dim=6, rot_dims=4, base=300.0), mlp(7, 1, 9, 0.5)),
    layer("latent_attention_2", mixer("latent_attention_2", 3, 8, 8, 24, 40, rot_dim=8), None),
], residual_mult=1.0, eps=1e-6, embed_scale=1.0)


def write_folder(folder, cfg, seed, dtype=torch.float32):
    """Random weights: matrices N(0, 1/sqrt(columns)) so that every product keeps its scale, norm weights around
    1, biases and sinks spread out so that leaving one out shows."""
    os.makedirs(folder, exist_ok=True)
    tensors = random_tensors(cfg, seed, std=1.0, norm_std=0.2, dtype=torch.float32)
    gen = torch.Generator().manual_seed(seed + 1)
    for name, t in tensors.items():
        if t.dim() == 2:
            tensors[name] = t * t.shape[1] ** -0.5
        elif name.endswith(".b"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.3
        elif name.endswith(".sink"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 2.0 + 1.0
        if name.endswith(".router"):
            tensors[name] = tensors[name] * 4.0           # clear choices: no test rests on a close call
    tensors = {k: v.to(dtype).contiguous() for k, v in tensors.items()}
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    save_file(tensors, os.path.join(folder, "model.safetensors"))
    return folder


def read_folder(folder):
    from safetensors import safe_open

    with open(os.path.join(folder, "config.json")) as f:
        cfg = json.load(f)
    w = {}
    with safe_open(os.path.join(folder, "model.safetensors"), framework="pt", device="cpu") as f:
        for name in f.keys():
            w[name] = f.get_tensor(name).to(torch.float32)
    return cfg, w
