"""Small Pedazen configurations and model folders with random weights, for the tests."""

from __future__ import annotations

import json
import os

import torch
from safetensors.torch import save_file

from tt_transformers_b200.weights import random_tensors


def lightning(heads, dim, vdim, decay):
    return {"type": "lightning", "mixer": {"heads": heads, "dim": dim, "vdim": vdim, "decay": list(decay)}}


def parallel(heads, kv_heads, dim, vdim, chunk, rot_dims, channels, blocks, taps, softcap=20.0, base=1000.0, scale=None):
    left = {"heads": heads, "kv_heads": kv_heads, "dim": dim, "vdim": vdim, "mask": {"size": chunk},
            "rot": {"base": base, "dims": rot_dims}, "scale": scale if scale is not None else dim ** -0.5, "softcap": softcap}
    return {"type": "parallel", "mixer": {"left": left, "right": {"width": channels, "blocks": blocks, "conv": taps}}}


def dense(ff):
    return {"kind": "dense", "ff": ff}


def moe(experts, top, ff, count, keep):
    return {"kind": "moe", "expert": {"ff": ff}, "router": {"experts": experts, "top": top, "groups": {"count": count, "keep": keep}}}


def layer(mixer, mlp):
    return dict(mixer, mlp=mlp)


def config(width, vocab, layers, loop, eps=1e-5, embed_scale=3.0):
    cfg = {"architecture": "Pedazen", "vocab": vocab, "width": width, "norm": {"eps": eps}, "embedding": {"scale": embed_scale},
           "layers": layers}
    if loop is not None:
        cfg["loop"] = {"start": loop[0], "stop": loop[1], "times": loop[2]}
    return cfg


# even sizes; a loop in the middle that runs three times; every kind of feed-forward and none
ALIGNED = config(128, 300, [
    layer(parallel(4, 2, 32, 16, chunk=24, rot_dims=16, channels=96, blocks=3, taps=3), dense(160)),
    layer(lightning(2, 48, 32, (0.9, 0.5)), moe(8, 2, 48, count=4, keep=2)),
    layer(parallel(6, 1, 16, 48, chunk=16, rot_dims=16, channels=64, blocks=2, taps=4, softcap=5.0), None),
    layer(lightning(3, 16, 64, (0.999, 0.97, 0.2)), moe(6, 3, 32, count=2, keep=1)),
], loop=(1, 3, 3))

# odd sizes and ones: one head, one block, one tap, one expert of one group, chunks of one and of seven positions,
# a rotation over a part of an odd-sized head, decays of 1 and 0, a loop that runs once and starts at the first layer
ODD = config(60, 131, [
    layer(lightning(1, 10, 6, (1.0,)), moe(1, 1, 20, count=1, keep=1)),
    layer(parallel(1, 1, 10, 7, chunk=7, rot_dims=6, channels=30, blocks=1, taps=1, softcap=50.0, base=300.0), moe(9, 1, 9, count=3, keep=3)),
    layer(parallel(5, 5, 6, 9, chunk=1, rot_dims=2, channels=20, blocks=5, taps=6, scale=0.7), dense(33)),
    layer(lightning(3, 5, 11, (0.0, 0.3, 0.8)), None),
], loop=(0, 2, 1), eps=1e-6, embed_scale=1.0)

# no loop at all, chunks longer than any test prompt (plain causal attention), taps longer than most portions
PLAIN = config(64, 200, [
    layer(parallel(2, 1, 24, 24, chunk=4096, rot_dims=24, channels=48, blocks=4, taps=9), moe(4, 2, 24, count=1, keep=1)),
    layer(lightning(2, 24, 24, (0.95, 0.8)), dense(96)),
], loop=None)


# head sizes that the tensor-core kernels take (attention with keys and values of 64, linear attention in chunks), chunks
# that end inside a key tile, a loop over both layers
TENSOR = config(128, 260, [
    layer(parallel(4, 2, 64, 64, chunk=40, rot_dims=32, channels=128, blocks=2, taps=4, softcap=15.0), moe(6, 2, 64, count=3, keep=2)),
    layer(lightning(2, 64, 64, (0.98, 0.7)), dense(192)),
], loop=(0, 2, 2))


def single(kind):
    """One layer with one mechanism and nothing beside it."""
    if kind == "lightning":
        layers = [layer(lightning(3, 20, 12, (0.99, 0.6, 0.9)), None)]
    elif kind == "parallel":
        layers = [layer(parallel(4, 2, 12, 20, chunk=10, rot_dims=8, channels=40, blocks=2, taps=4), None)]
    elif kind == "dense":
        layers = [layer(lightning(1, 8, 8, (0.5,)), dense(72))]
    else:
        layers = [layer(lightning(1, 8, 8, (0.5,)), moe(12, 3, 20, count=3, keep=2))]
    return config(48, 97, layers, loop=None)


def write_folder(folder, cfg, seed, dtype=torch.float32):
    """Random weights: matrices N(0, 1/sqrt(columns)) so that every product keeps its scale; norm weights that
    are stored around zero around zero, plain ones around one; biases, sinks, pass vectors and decay rates spread
    out so that leaving one out shows; routers with clear choices."""
    os.makedirs(folder, exist_ok=True)
    tensors = random_tensors(cfg, seed, std=1.0, norm_std=0.2, dtype=torch.float32)
    gen = torch.Generator().manual_seed(seed + 1)
    for name, t in tensors.items():
        if name.endswith(("norm1", "final.norm")):
            tensors[name] = t - 1.0
        elif name.endswith(".b"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.3
        elif name.endswith(".sink"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 2.0 + 1.0
        elif name.endswith(".lam"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 1.5 - 1.0
        elif name.endswith(".conv"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.5
        elif name == "loop.step":
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.5
        elif t.dim() >= 2:
            tensors[name] = t * t.shape[-1] ** -0.5
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
