"""A plain, slow implementation of the Pedazen decoder: one function per mechanism, whole sequences at once,
float64 unless told otherwise. It shares no code with the package; the tests compare the engine with it.

A model is (config dictionary, {tensor name: tensor}). Weights are [out, in] and applied as W x.

    embedding:   x = E[token] * scale
    layer:       h = rms(x) * (1 + w);  x = x + (mixer(h) + ff(h))
    loop:        layers start .. stop-1 run `times` times with the same weights and a state of their own per pass;
                 before every pass but the first x += x0 (the embedding's output); before every pass x += step[pass]
    output:      logits = E (rms(x) * (1 + w_final))
"""

import math

import torch

F = torch.float64


def rms(x, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)


def gelu_tanh(z):
    return 0.5 * z * (1 + torch.tanh(math.sqrt(2 / math.pi) * (z + 0.044715 * z ** 3)))


def silu(z):
    return z * torch.sigmoid(z)


def lightning_mixer(h, w, p, m, eps):
    """h [T, width]. Per head: S_t = decay S_(t-1) + k_t v_t^T, o_t = S_t^T q_t; the heads' outputs together are
    RMS-normed (plain weight), gated by sigmoid(W_g h) and projected."""
    T = h.shape[0]
    H, D, V = m["heads"], m["dim"], m["vdim"]
    q = silu(h @ w[p + "q"].T).view(T, H, D)
    k = silu(h @ w[p + "k"].T).view(T, H, D)
    v = silu(h @ w[p + "v"].T).view(T, H, V)
    out = torch.zeros(T, H, V, dtype=h.dtype)
    for head in range(H):
        S = torch.zeros(D, V, dtype=h.dtype)
        for t in range(T):
            S = m["decay"][head] * S + torch.outer(k[t, head], v[t, head])
            out[t, head] = S.T @ q[t, head]
    o = rms(out.reshape(T, H * V), eps) * w[p + "norm"]
    return (o * torch.sigmoid(h @ w[p + "g"].T)) @ w[p + "o"].T


def rotate(x, positions, dims, base):
    """x [T, heads, dim]: element i of the first `dims` is paired with element i + dims/2."""
    half = dims // 2
    freq = base ** (-2.0 * torch.arange(half, dtype=x.dtype) / dims)
    angle = positions.to(x.dtype)[:, None] * freq[None, :]
    cos, sin = torch.cos(angle)[:, None, :], torch.sin(angle)[:, None, :]
    u, v = x[..., :half], x[..., half:dims]
    return torch.cat([u * cos - v * sin, v * cos + u * sin, x[..., dims:]], -1)


def chunked_sink_attention(h, w, p, m, eps):
    """Grouped-query attention with per-head RMS norms on q and k, a partial rotation, capped scores, a mask
    that lets position i see j <= i of its own chunk only, and a sink per head in the softmax's denominator."""
    T = h.shape[0]
    H, G, D, V = m["heads"], m["kv_heads"], m["dim"], m["vdim"]
    q = (h @ w[p + "q"].T).view(T, H, D)
    k = (h @ w[p + "k"].T).view(T, G, D)
    v = (h @ w[p + "v"].T).view(T, G, V)
    q = rms(q, eps) * w[p + "q.norm"]
    k = rms(k, eps) * w[p + "k.norm"]
    pos = torch.arange(T)
    q = rotate(q, pos, m["rot"]["dims"], m["rot"]["base"])
    k = rotate(k, pos, m["rot"]["dims"], m["rot"]["base"])
    size, cap = m["mask"]["size"], m["softcap"]
    out = torch.zeros(T, H, V, dtype=h.dtype)
    for head in range(H):
        g = head // (H // G)
        for i in range(T):
            lo = (i // size) * size
            s = (k[lo:i + 1, g] @ q[i, head]) * m["scale"]
            s = cap * torch.tanh(s / cap)
            top = max(float(s.max()), float(w[p + "sink"][head]))
            e = torch.exp(s - top)
            denom = e.sum() + math.exp(float(w[p + "sink"][head]) - top)
            out[i, head] = (e / denom) @ v[lo:i + 1, g]
    return out.reshape(T, H * V) @ w[p + "o"].T


def recurrent_block(h, w, p, m):
    """Two branches: y = gelu(W_y h + b) and u = causal per-channel convolution of (W_x h + b); a gated linear
    recurrence over u with decays from a block-diagonal gate; output W_o (S * y)."""
    T = h.shape[0]
    C, B, taps = m["width"], m["blocks"], m["conv"]
    y = gelu_tanh(h @ w[p + "y"].T + w[p + "y.b"])
    xin = h @ w[p + "x"].T + w[p + "x.b"]
    padded = torch.cat([torch.zeros(taps - 1, C, dtype=h.dtype), xin], 0)
    u = torch.zeros(T, C, dtype=h.dtype) + w[p + "conv.b"]
    for j in range(taps):
        u = u + padded[j:j + T] * w[p + "conv"][:, j]
    ub = u.view(T, B, C // B)
    r = torch.sigmoid(torch.einsum("boi,tbi->tbo", w[p + "ra"], ub) + w[p + "ra.b"]).reshape(T, C)
    i = torch.sigmoid(torch.einsum("boi,tbi->tbo", w[p + "ri"], ub) + w[p + "ri.b"]).reshape(T, C)
    log_a = -8.0 * r * torch.nn.functional.softplus(w[p + "lam"])
    a = torch.exp(log_a)
    S = torch.zeros(C, dtype=h.dtype)
    out = torch.zeros(T, C, dtype=h.dtype)
    for t in range(T):
        S = a[t] * S + torch.sqrt(1 - a[t] ** 2) * i[t] * u[t]
        out[t] = S
    return (out * y) @ w[p + "o"].T


def parallel_mixer(h, w, p, m, eps):
    left = chunked_sink_attention(h, w, p + "left.", m["left"], eps)
    right = recurrent_block(h, w, p + "right.", m["right"])
    return 0.5 * (rms(left, eps) * w[p + "left.out"] + rms(right, eps) * w[p + "right.out"])


def dense_ff(h, w, p):
    return (gelu_tanh(h @ w[p + "gate"].T) * (h @ w[p + "up"].T)) @ w[p + "down"].T


def route(h, w_router, r):
    """-> (chosen experts [T, top], weights [T, top]): softmax over all experts, only experts of the `keep` groups
    with the largest best score may be chosen, the chosen scores are divided by their sum."""
    s = torch.softmax(h @ w_router.T, -1)
    T, E = s.shape
    count, keep = r["groups"]["count"], r["groups"]["keep"]
    best = s.view(T, count, E // count).max(-1).values
    kept = best.topk(keep, -1).indices
    allowed = torch.zeros(T, count, dtype=torch.bool)
    allowed.scatter_(1, kept, True)
    masked = torch.where(allowed.repeat_interleave(E // count, 1), s, torch.full_like(s, -1.0))
    choice = masked.topk(r["top"], -1).indices
    chosen = s.gather(1, choice)
    return choice, chosen / (chosen.sum(-1, keepdim=True) + 1e-20)


def expert(h, w, p):
    return (torch.relu(h @ w[p + "up"].T) ** 2) @ w[p + "down"].T


def moe_ff(h, w, p, f):
    choice, weight = route(h, w[p + "router"], f["router"])
    out = torch.zeros_like(h)
    for t in range(h.shape[0]):
        for j in range(choice.shape[1]):
            out[t] += weight[t, j] * expert(h[t:t + 1], w, f"{p}e{int(choice[t, j])}.")[0]
    return out


def layer_order(cfg):
    """[(layer, pass number or None)] in running order; the pass number is given at the first layer of a pass."""
    n, loop = len(cfg["layers"]), cfg.get("loop")
    if not loop:
        return [(i, None) for i in range(n)]
    order = [(i, None) for i in range(loop["start"])]
    for t in range(loop["times"]):
        order += [(i, t if i == loop["start"] else None) for i in range(loop["start"], loop["stop"])]
    return order + [(i, None) for i in range(loop["stop"], n)]


def forward(cfg, weights, tokens, dtype=F, streams=None):
    """Logits [T, vocab] of one sequence. `streams`, a list, receives x after every layer run."""
    w = {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in weights.items()}
    eps = cfg["norm"]["eps"]
    x0 = w["embed"][torch.as_tensor(tokens, dtype=torch.long)] * cfg["embedding"]["scale"]
    x = x0.clone()
    for i, t in layer_order(cfg):
        layer, p = cfg["layers"][i], f"l{i}."
        if t is not None:
            if t > 0:
                x = x + x0
            x = x + w["loop.step"][t]
        h = rms(x, eps) * (1 + w[p + "norm1"])
        if layer["type"] == "lightning":
            mixed = lightning_mixer(h, w, p + "mix.", layer["mixer"], eps)
        else:
            mixed = parallel_mixer(h, w, p + "mix.", layer["mixer"], eps)
        f = layer["mlp"]
        if f is None:
            ff = 0
        elif f["kind"] == "dense":
            ff = dense_ff(h, w, p + "mlp.")
        else:
            ff = moe_ff(h, w, p + "mlp.", f)
        x = x + (mixed + ff)
        if streams is not None:
            streams.append(x.clone())
    return (rms(x, eps) * (1 + w["final.norm"])) @ w["embed"].T
