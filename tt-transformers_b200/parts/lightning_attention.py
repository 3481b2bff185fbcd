"""Linear attention with a fixed decay per head and a matrix state per request.

    q = silu(W_q h), k = silu(W_k h) [heads, dim];  v = silu(W_v h) [heads, vdim]
    S_t = decay_h S_(t-1) + k_t v_t^T;   o_t = S_t^T q_t          (per head; no other scale)
    out = W_o (rms(o over all heads) * g_norm * sigmoid(W_g h))

The state S [heads, dim, vdim] is float32, starts at zero and lives in a slot of the cache manager per live
request; a step's tokens continue from what the step before left. The four projections of one input run as
one product; the activations, the recurrence, the norm and the gate are float32.
"""

from __future__ import annotations

import torch

from .base import Mixer, SlotState, TensorSpec, register_part


class LightningAttention(Mixer):
    graph_safe = True

    def __init__(self, width: int, heads: int, dim: int, vdim: int, decay, eps: float, prefix: str, position=None):
        self.width, self.heads, self.dim, self.vdim = int(width), int(heads), int(dim), int(vdim)
        self.decay = tuple(float(d) for d in decay)
        self.eps, self.prefix = float(eps), prefix
        if len(self.decay) != self.heads:
            raise ValueError(f"{len(self.decay)} decays for {self.heads} heads")
        if any(not 0.0 <= d <= 1.0 for d in self.decay):
            raise ValueError("a decay must lie between 0 and 1")

    def tensor_specs(self):
        p, H = self.prefix, self.heads
        return [TensorSpec(p + "q", (H * self.dim, self.width)), TensorSpec(p + "k", (H * self.dim, self.width)),
                TensorSpec(p + "v", (H * self.vdim, self.width)), TensorSpec(p + "g", (H * self.vdim, self.width)),
                TensorSpec(p + "o", (self.width, H * self.vdim)), TensorSpec(p + "norm", (H * self.vdim,))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        self.w_in = runtime.matrix(torch.cat([tensors[p + "q"], tensors[p + "k"], tensors[p + "v"], tensors[p + "g"]], 0))
        self.w_o = runtime.matrix(tensors[p + "o"])
        self.norm = tensors[p + "norm"].to(device=runtime.device, dtype=torch.float32).contiguous()
        self.decays = torch.tensor(self.decay, dtype=torch.float32, device=runtime.device)

    def cache_request(self):
        return SlotState((self.heads, self.dim, self.vdim), torch.float32)

    def forward(self, x, batch, cache, write_cache=True):
        k = self.runtime.kernels
        H, D, V = self.heads, self.dim, self.vdim
        proj = k.linear(x, self.w_in)                                   # [T, q | k | v | g]
        o = k.lightning_attention(proj, batch, cache, H, D, V, self.decays, write_cache)      # float32 [T, H * V]
        gated = k.gated_rmsnorm(o, self.norm, self.eps, proj[:, 2 * H * D + H * V:], self.runtime.dtype)
        return k.linear(gated, self.w_o)


register_part("mixer", "lightning_attention", LightningAttention)
