"""Plain, slow Bozavik forward pass: the oracle that the engine is compared with.

Whole sequences, no cache, no paging, 32-bit floats on the CPU, one function per mechanism,
written from the design's equations. It shares no code with the package.

The design: a scaled embedding; layers of the form
    x <- x + m * LN_1b(mixer(LN_1(x)));   x <- x + m * LN_2b(ff(LN_2(x)))
with layer norms that carry a weight and a bias; two mixers, both attention over a cached
low-rank latent (one without positions and with a learned sink in the softmax's denominator and
an element-wise output gate, one with a rotated key part shared by all heads and one gate number
per head); a routed feed-forward of clamped experts plus a gated shared expert; a final layer
norm and a linear head.
"""

from __future__ import annotations

import math

import torch


# ---------------------------------------------------------------------------- norms
def layer_norm(x, weight, bias, eps):
    """(x - mean) / sqrt(var + eps) * w + b, the variance being the mean squared deviation."""
    mean = x.mean(dim=-1, keepdim=True)
    dev = x - mean
    var = (dev * dev).mean(dim=-1, keepdim=True)
    return dev / torch.sqrt(var + eps) * weight + bias


def rms_norm(x, weight, eps):
    """x / sqrt(mean(x^2) + eps) * w."""
    return x / torch.sqrt((x * x).mean(dim=-1, keepdim=True) + eps) * weight


# ---------------------------------------------------------------------------- rotation
def rotate_halves(x, positions, base, dims):
    """x [T, ..., D]: the first `dims` elements of the last axis are rotated, element i with element
    i + dims/2, by the angle position * base^(-2i/dims); the rest passes unchanged."""
    half = dims // 2
    out = x.clone()
    for i in range(half):
        freq = base ** (-2.0 * i / dims)
        angle = positions.to(torch.float64) * freq
        cos, sin = torch.cos(angle).float(), torch.sin(angle).float()
        shape = [-1] + [1] * (x.dim() - 2)
        cos, sin = cos.view(shape), sin.view(shape)
        u, v = x[..., i], x[..., i + half]
        out[..., i] = u * cos - v * sin
        out[..., i + half] = v * cos + u * sin
    return out


# ---------------------------------------------------------------------------- the mixers
def latent_attention(mixer, w, p, h, eps, positions=None):
    """Both mixers. mixer: the layer's `mixer` dictionary; p: the tensor prefix ('l3.mix.'); h [T, width].

    c_q = RMS(W_dq h); q = W_uq c_q, per head [dim | rot_dim]. W_dkv h = [latent rows | rot_dim rows];
    c = RMS(latent rows); the rot_dim rows, rotated, are one key part shared by all heads. Per head
    k = W_uk c, v = W_uv c; score = (q_plain . k + q_rot . k_rot) * scale; causal softmax, with exp(sink_h)
    added to the denominator where the mixer has a sink; the heads' outputs are gated by sigmoid(W_g h)
    (as many gate rows as output elements, or one per head) and projected by W_o."""
    T = h.shape[0]
    H, D, V, R = mixer["heads"], mixer["dim"], mixer["vdim"], mixer["kv_rank"]
    rot = int(mixer.get("rot_dim", 0) or 0)
    positions = torch.arange(T) if positions is None else positions
    c_q = rms_norm(h @ w[p + "dq"].T, w[p + "dq.norm"], eps)
    q = (c_q @ w[p + "uq"].T).view(T, H, D + rot)
    down = h @ w[p + "dkv"].T
    c = rms_norm(down[:, :R], w[p + "dkv.norm"], eps)
    k = (c @ w[p + "uk"].T).view(T, H, D)
    v = (c @ w[p + "uv"].T).view(T, H, V)
    scores = torch.einsum("thd,shd->hts", q[..., :D], k)
    if rot:
        base, dims = mixer["rot"]["base"], mixer["rot"]["dims"]
        q_rot = rotate_halves(q[..., D:], positions, base, dims)
        k_rot = rotate_halves(down[:, R:], positions, base, dims)
        scores = scores + torch.einsum("thd,sd->hts", q_rot, k_rot)
    scores = scores * mixer["scale"]
    visible = torch.arange(T)[None, :] <= torch.arange(T)[:, None]
    scores = scores.masked_fill(~visible, float("-inf"))
    if (p + "sink") in w:
        # the sink is one more column of the softmax that has no value: its weight is dropped afterwards
        sink = w[p + "sink"].view(H, 1, 1).expand(H, T, 1)
        weights = torch.softmax(torch.cat([scores, sink], dim=-1), dim=-1)[..., :T]
    else:
        weights = torch.softmax(scores, dim=-1)
    out = torch.einsum("hts,shv->thv", weights, v)
    gate = torch.sigmoid(h @ w[p + "g"].T)
    if gate.shape[1] == H:
        out = out * gate[:, :, None]
        out = out.reshape(T, H * V)
    else:
        out = out.reshape(T, H * V) * gate
    return out @ w[p + "o"].T


# ---------------------------------------------------------------------------- the feed-forward
def clamped_expert(h, gate, up, down, limit):
    """g = min(W_gate h, limit); u = clamp(W_up h, -limit, limit); W_down (g sigmoid(1.702 g) (u + 1))."""
    g = torch.clamp(h @ gate.T, max=limit)
    u = torch.clamp(h @ up.T, min=-limit, max=limit)
    return (g * torch.sigmoid(1.702 * g) * (u + 1.0)) @ down.T


def routed_feed_forward(mlp, w, p, h):
    """Router logits W_router h; the `top` largest are chosen; their weights are the softmax over the chosen
    logits; the output is the weighted sum of the chosen experts, plus the shared expert times sigmoid(W_sg h)."""
    T = h.shape[0]
    experts, top = mlp["router"]["experts"], mlp["router"]["top"]
    logits = h @ w[p + "router"].T
    out = torch.zeros(T, w[p + "e0.down"].shape[0])
    for t in range(T):
        order = sorted(range(experts), key=lambda e: (-float(logits[t, e]), e))[:top]
        chosen = torch.stack([logits[t, e] for e in order])
        weights = torch.softmax(chosen, dim=0)
        for weight, e in zip(weights, order):
            q = f"{p}e{e}."
            out[t] += weight * clamped_expert(h[t:t + 1], w[q + "gate"], w[q + "up"], w[q + "down"], mlp["expert"]["limit"])[0]
    if mlp.get("shared"):
        q = p + "shared."
        shared = clamped_expert(h, w[q + "gate"], w[q + "up"], w[q + "down"], mlp["shared"]["limit"])
        out = out + shared * torch.sigmoid(h @ w[q + "sg"].T)
    return out


# ---------------------------------------------------------------------------- the model
def forward(config, w, tokens, positions=None, keep_layers=False):
    """Logits [T, vocab] of a whole sequence (and, with keep_layers, the residual stream after every layer)."""
    eps, m = config["norm"]["eps"], config["residual_mult"]
    x = w["embed"][torch.as_tensor(tokens)] * config["embedding"]["scale"]
    kept = []
    for i, layer in enumerate(config["layers"]):
        p = f"l{i}."
        if layer["type"] not in ("latent_attention", "latent_attention_2"):
            raise ValueError(f"unknown layer type {layer['type']}")
        h = layer_norm(x, w[p + "norm1"], w[p + "norm1.b"], eps)
        mixed = latent_attention(layer["mixer"], w, p + "mix.", h, eps, positions)
        x = x + m * layer_norm(mixed, w[p + "norm1b"], w[p + "norm1b.b"], eps)
        if layer.get("mlp") is not None:
            h = layer_norm(x, w[p + "norm2"], w[p + "norm2.b"], eps)
            x = x + m * layer_norm(routed_feed_forward(layer["mlp"], w, p + "mlp.", h), w[p + "norm2b"], w[p + "norm2b.b"], eps)
        kept.append(x.clone())
    logits = layer_norm(x, w["final.norm"], w["final.norm.b"], eps) @ w["head"].T
    return (logits, torch.stack(kept)) if keep_layers else logits


def softmax_row_with_sink(scores, sink):
    """One row of attention weights whose denominator also holds exp(sink): they sum to less than one."""
    top = max(float(scores.max()), float(sink))
    e = torch.exp(scores - top)
    return e / (e.sum() + math.exp(float(sink) - top))
