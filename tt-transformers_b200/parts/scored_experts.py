"""A routed feed-forward whose router scores every expert by itself and whose score multiplies the expert's input.

    s = sigmoid(W_r h) (float32; `scores` "sigmoid"), the `top` largest are chosen, the lower index among equals
    the chosen experts' scores are their weights as they are (not renormalised)
    expert: y = W_down (silu(W_gate u) * (W_up u)), no biases
    out = sum_j expert_j(s_j * h), float32, summed in the order of the router's choice

Because the weight stands before the expert's activation it cannot be pulled out of the expert. Tokens are grouped
by expert on the device, as for the other routed feed-forwards of this package.
"""

from __future__ import annotations

import torch

from .base import FeedForward, TensorSpec, register_part


class ScoredExperts(FeedForward):
    graph_safe = True

    def __init__(self, width: int, experts: int, top: int, inter: int, prefix: str, scores: str = "sigmoid"):
        self.width, self.experts, self.top, self.inter = int(width), int(experts), int(top), int(inter)
        self.prefix, self.scores = prefix, scores
        if not 1 <= self.top <= self.experts:
            raise ValueError(f"top ({top}) must lie between 1 and the number of experts ({experts})")
        if scores != "sigmoid":
            raise ValueError(f"scores {scores!r} is not built; known: ['sigmoid']")

    def tensor_specs(self):
        p = self.prefix
        specs = [TensorSpec(p + "router", (self.experts, self.width))]
        for e in range(self.experts):
            specs += [TensorSpec(f"{p}e{e}.gate", (self.inter, self.width)), TensorSpec(f"{p}e{e}.up", (self.inter, self.width)),
                      TensorSpec(f"{p}e{e}.down", (self.width, self.inter))]
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        self.w_router = tensors[p + "router"].to(device=runtime.device, dtype=torch.float32).contiguous()
        self.w_gate_up = runtime.matrix(torch.stack(
            [torch.cat([tensors[f"{p}e{e}.gate"], tensors[f"{p}e{e}.up"]], 0) for e in range(self.experts)]))
        self.w_down = runtime.matrix(torch.stack([tensors[f"{p}e{e}.down"] for e in range(self.experts)]))

    def forward(self, x, batch):
        k = self.runtime.kernels
        choice, weight, _ = k.route_top(x, self.w_router, self.experts, self.top, False, scores=self.scores)
        return k.input_weighted_experts(x, choice, weight, self.w_gate_up, self.w_down)       # float32 [T, width]


register_part("feed_forward", "scored_experts", ScoredExperts)
