"""A routed feed-forward whose router scores all experts and may choose from the best groups only.

    s = softmax(W_r h) over all experts (float32)
    experts form `groups` equal groups of neighbours; a group's score is its largest s; only experts of the
    `keep` best groups can be chosen (groups = keep = 1: no restriction)
    the `top` largest s among them are chosen; their weights are s / (sum of the chosen s + 1e-20)
    expert: y = W_down act(W_up h), act = relu(z)^2 (or another registered name), no biases, no gate
    out = sum_j weight_j * expert_j(h), float32, summed in the order of the router's choice

Tokens are grouped by expert on the device, as for the other routed feed-forward of this package.
"""

from __future__ import annotations

import torch

from .base import FeedForward, TensorSpec, register_part

NORMALISER_FLOOR = 1e-20


class GroupedExperts(FeedForward):
    graph_safe = True

    def __init__(self, width: int, experts: int, top: int, inter: int, prefix: str, groups: int = 1, keep: int = 1,
                 activation: str = "relu2"):
        self.width, self.experts, self.top, self.inter = int(width), int(experts), int(top), int(inter)
        self.groups, self.keep, self.prefix, self.activation = int(groups), int(keep), prefix, activation
        if not 1 <= self.top <= self.experts:
            raise ValueError(f"top ({top}) must lie between 1 and the number of experts ({experts})")
        if self.groups < 1 or self.experts % self.groups:
            raise ValueError(f"{experts} experts do not split into {groups} equal groups")
        if not 1 <= self.keep <= self.groups:
            raise ValueError(f"keep ({keep}) must lie between 1 and the number of groups ({groups})")
        if self.keep * (self.experts // self.groups) < self.top:
            raise ValueError(f"{keep} groups of {self.experts // self.groups} experts cannot give {top} choices")
        if activation != "relu2":
            raise ValueError(f"activation {activation!r} is not built; known: ['relu2']")

    def tensor_specs(self):
        p = self.prefix
        specs = [TensorSpec(p + "router", (self.experts, self.width))]
        for e in range(self.experts):
            specs += [TensorSpec(f"{p}e{e}.up", (self.inter, self.width)), TensorSpec(f"{p}e{e}.down", (self.width, self.inter))]
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        self.w_router = tensors[p + "router"].to(device=runtime.device, dtype=torch.float32).contiguous()
        self.w_up = runtime.matrix(torch.stack([tensors[f"{p}e{e}.up"] for e in range(self.experts)]))
        self.w_down = runtime.matrix(torch.stack([tensors[f"{p}e{e}.down"] for e in range(self.experts)]))

    def forward(self, x, batch):
        k = self.runtime.kernels
        choice, weight = k.route_grouped(x, self.w_router, self.experts, self.top, self.groups, self.keep, NORMALISER_FLOOR)
        return k.plain_experts(x, choice, weight, self.w_up, self.w_down, self.activation)       # float32 [T, width]


register_part("feed_forward", "grouped_experts", GroupedExperts)
