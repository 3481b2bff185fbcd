"""A routed feed-forward: many small gated experts of which each token uses a few, plus an optional shared one.

Router: logits z = W_r h in float32; the `top` largest are chosen (the lower index among equals) and weighted
by the softmax over the chosen logits only. Expert (no biases), with `limit` L and the constant a = 1.702:
    g = min(W_gate h, L);  u = clamp(W_up h, -L, L);  y = W_down (g * sigmoid(a g) * (u + 1)).
The output is the weighted sum of the chosen experts' outputs, in float32, summed in the order of the
router's choice whatever else the batch holds. The shared expert has the same form with sizes and a limit of
its own; it runs for every token and is multiplied by sigmoid(w_sg . h), one number per token.

Tokens are grouped by expert on the device (no host read, so steps can be captured): a counting kernel lays
out the (token, choice) pairs expert by expert, both products of the experts run over those groups, and the
last kernel sums each token's pairs.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import FeedForward, TensorSpec, register_part

GLU_ALPHA = 1.702


class RoutedExperts(FeedForward):
    graph_safe = True

    def __init__(self, width: int, experts: int, top: int, inter: int, limit: float, prefix: str,
                 shared_inter: Optional[int] = None, shared_limit: Optional[float] = None, alpha: float = GLU_ALPHA):
        self.width, self.experts, self.top, self.inter = int(width), int(experts), int(top), int(inter)
        self.limit, self.prefix, self.alpha = float(limit), prefix, float(alpha)
        self.shared_inter = None if shared_inter is None else int(shared_inter)
        self.shared_limit = float(shared_limit) if shared_limit is not None else self.limit
        if not 1 <= self.top <= self.experts:
            raise ValueError(f"top ({top}) must lie between 1 and the number of experts ({experts})")

    def tensor_specs(self):
        p = self.prefix
        specs = [TensorSpec(p + "router", (self.experts, self.width))]
        for e in range(self.experts):
            specs += [TensorSpec(f"{p}e{e}.gate", (self.inter, self.width)), TensorSpec(f"{p}e{e}.up", (self.inter, self.width)),
                      TensorSpec(f"{p}e{e}.down", (self.width, self.inter))]
        if self.shared_inter is not None:
            s = self.shared_inter
            specs += [TensorSpec(p + "shared.gate", (s, self.width)), TensorSpec(p + "shared.up", (s, self.width)),
                      TensorSpec(p + "shared.down", (self.width, s)), TensorSpec(p + "shared.sg", (1, self.width))]
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        router = [tensors[p + "router"]] + ([tensors[p + "shared.sg"]] if self.shared_inter is not None else [])
        # the router's rows and, after them, the shared expert's gate row: float32, one small product
        self.w_router = torch.cat(router, 0).to(device=runtime.device, dtype=torch.float32).contiguous()
        self.w_gate_up = runtime.matrix(torch.stack(
            [torch.cat([tensors[f"{p}e{e}.gate"], tensors[f"{p}e{e}.up"]], 0) for e in range(self.experts)]))
        self.w_down = runtime.matrix(torch.stack([tensors[f"{p}e{e}.down"] for e in range(self.experts)]))
        if self.shared_inter is not None:
            self.ws_gate_up = runtime.matrix(torch.cat([tensors[p + "shared.gate"], tensors[p + "shared.up"]], 0))
            self.ws_down = runtime.matrix(tensors[p + "shared.down"])

    def forward(self, x, batch):
        k = self.runtime.kernels
        shared = self.shared_inter is not None
        choice, weight, shared_gate = k.route_top(x, self.w_router, self.experts, self.top, shared)
        shared_expert = (self.ws_gate_up, self.ws_down, self.shared_limit) if shared else None
        return k.routed_experts(x, choice, weight, self.w_gate_up, self.w_down, self.limit, self.alpha,
                                shared_expert, shared_gate)       # float32 [T, width]


register_part("feed_forward", "routed_experts", RoutedExperts)
