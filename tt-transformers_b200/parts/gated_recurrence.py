"""A recurrent block: a gated linear recurrence per channel behind a short causal convolution, beside a gate branch.

    y = gelu_tanh(W_y h + b_y);   x' = W_x h + b_x                                  (`channels` each)
    u_t = b_c + sum_j c[:, j] x'_(t - taps + 1 + j)                                 (per channel; zeros before the start)
    per block b of channels:  r = sigmoid(R_b u_b + r_b),  i = sigmoid(I_b u_b + i_b)   (block-diagonal gates)
    a = exp(-DECAY_SHARPNESS r softplus(lam));   S_t = a S_(t-1) + sqrt(1 - a^2) (i * u_t)
    out = W_o (S_t * y)

The recurrence follows De et al., "Griffin: Mixing Gated Linear Recurrences with Local Attention for Efficient
Language Models" (2024). The state S (float32) and the convolution's last taps - 1 inputs live in a slot per
live request, zero at the start; the first token has no special case. Gates, decays, the recurrence and its
state are float32; the gates' block products accumulate in float32 and leave float32.
"""

from __future__ import annotations

import torch

from .base import Mixer, RecurrentState, TensorSpec, register_part

DECAY_SHARPNESS = 8.0


class GatedRecurrence(Mixer):
    graph_safe = True

    def __init__(self, width: int, channels: int, blocks: int, taps: int, prefix: str, sharpness: float = DECAY_SHARPNESS,
                 position=None):
        self.width, self.channels, self.blocks, self.taps = int(width), int(channels), int(blocks), int(taps)
        self.prefix, self.sharpness = prefix, float(sharpness)
        if self.channels % self.blocks:
            raise ValueError(f"{channels} channels do not split into {blocks} equal blocks")
        if self.taps < 1:
            raise ValueError("the convolution needs at least one tap")

    def tensor_specs(self):
        p, C, B = self.prefix, self.channels, self.blocks
        s = C // B
        return [TensorSpec(p + "y", (C, self.width)), TensorSpec(p + "y.b", (C,)), TensorSpec(p + "x", (C, self.width)),
                TensorSpec(p + "x.b", (C,)), TensorSpec(p + "conv", (C, self.taps)), TensorSpec(p + "conv.b", (C,)),
                TensorSpec(p + "ra", (B, s, s)), TensorSpec(p + "ra.b", (B, s)), TensorSpec(p + "ri", (B, s, s)),
                TensorSpec(p + "ri.b", (B, s)), TensorSpec(p + "lam", (C,)), TensorSpec(p + "o", (self.width, C))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        f32 = dict(device=runtime.device, dtype=torch.float32)
        self.w_in = runtime.matrix(torch.cat([tensors[p + "y"], tensors[p + "x"]], 0))           # [2 C, width]
        self.b_in = torch.cat([tensors[p + "y.b"], tensors[p + "x.b"]], 0).to(**f32).contiguous()
        self.conv = tensors[p + "conv"].to(**f32).contiguous()                                    # [C, taps]
        self.conv_b = tensors[p + "conv.b"].to(**f32).contiguous()
        # per block the rows of the decay gate followed by the rows of the input gate: one product gives both
        self.w_gates = runtime.matrix(torch.cat([tensors[p + "ra"], tensors[p + "ri"]], 1))       # [B, 2 s, s]
        self.b_gates = torch.cat([tensors[p + "ra.b"], tensors[p + "ri.b"]], 1).to(**f32).contiguous()   # [B, 2 s]
        # softplus(lam) does not depend on the token: once, in float32
        self.rate = torch.nn.functional.softplus(tensors[p + "lam"].to(torch.float32)).mul(self.sharpness).to(**f32).contiguous()
        self.w_o = runtime.matrix(tensors[p + "o"])

    def cache_request(self):
        return RecurrentState(self.channels, self.taps)

    @property
    def input_weight(self):
        return self.w_in

    @input_weight.setter
    def input_weight(self, rows):
        self.w_in = rows

    def forward(self, x, batch, cache, write_cache=True, projected=None):
        k = self.runtime.kernels
        C, B = self.channels, self.blocks
        yx = projected if projected is not None else k.linear(x, self.w_in)                                            # [T, y | x'] without their biases
        if batch.max_seg_len == 1 and (C // B) * 12 <= 48 * 1024:
            # decoded tokens: convolution, gates and recurrence in one kernel
            mixed = k.recurrent_token(yx, self.b_in, self.conv, self.conv_b, self.w_gates, self.b_gates, self.rate, batch, cache,
                                      write_cache)
            return k.linear(mixed, self.w_o)
        u = k.causal_conv(yx[:, C:], self.b_in[C:], self.conv, self.conv_b, batch, cache)          # [T, C]
        gates = k.heads_linear(u.view(-1, B, C // B), self.w_gates, out_dtype=torch.float32)      # [T, B, 2 s]
        mixed = k.gated_recurrence(u, gates, self.b_gates, self.rate, yx, self.b_in, batch, cache, write_cache)
        return k.linear(mixed, self.w_o)


register_part("mixer", "gated_recurrence", GatedRecurrence)
