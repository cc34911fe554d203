"""A routed feed-forward whose router scores every expert by itself and chooses with a correction per expert.

    s = sigmoid(W_r h)  (float32);  the `top` experts with the largest s + correction are chosen (the lower index among
    equals); the correction steers the choice only (a load-balancing bias that training moves instead of an auxiliary
    loss): the weights are the chosen experts' s, divided by their sum (+ 1e-20) and multiplied by `scale`
    expert: y = W_down (silu(W_gate h) * (W_up h)), no biases
    out = sum_j weight_j * expert_j(h) + shared(h), float32, summed in the order of the router's choice; the shared
    expert (optional, same form, a size of its own) runs for every token and has no gate

Tokens are grouped by expert on the device, as for the other routed feed-forwards of this package.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import FeedForward, TensorSpec, register_part

NORMALISER_FLOOR = 1e-20


class CorrectedExperts(FeedForward):
    graph_safe = True

    def __init__(self, width: int, experts: int, top: int, inter: int, prefix: str, scale: float = 1.0,
                 shared_inter: Optional[int] = None):
        self.width, self.experts, self.top, self.inter = int(width), int(experts), int(top), int(inter)
        self.prefix, self.scale = prefix, float(scale)
        self.shared_inter = None if shared_inter is None else int(shared_inter)
        if not 1 <= self.top <= self.experts:
            raise ValueError(f"top ({top}) must lie between 1 and the number of experts ({experts})")

    def tensor_specs(self):
        p = self.prefix
        specs = [TensorSpec(p + "router", (self.experts, self.width)), TensorSpec(p + "correction", (self.experts,))]
        for e in range(self.experts):
            specs += [TensorSpec(f"{p}e{e}.gate", (self.inter, self.width)), TensorSpec(f"{p}e{e}.up", (self.inter, self.width)),
                      TensorSpec(f"{p}e{e}.down", (self.width, self.inter))]
        if self.shared_inter is not None:
            s = self.shared_inter
            specs += [TensorSpec(p + "shared.gate", (s, self.width)), TensorSpec(p + "shared.up", (s, self.width)),
                      TensorSpec(p + "shared.down", (self.width, s))]
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        f32 = dict(device=runtime.device, dtype=torch.float32)
        self.w_router = tensors[p + "router"].to(**f32).contiguous()
        self.correction = tensors[p + "correction"].to(**f32).contiguous()
        self.w_gate_up = runtime.matrix(torch.stack(
            [torch.cat([tensors[f"{p}e{e}.gate"], tensors[f"{p}e{e}.up"]], 0) for e in range(self.experts)]))
        self.w_down = runtime.matrix(torch.stack([tensors[f"{p}e{e}.down"] for e in range(self.experts)]))
        self.shared = None
        if self.shared_inter is not None:
            self.shared = (runtime.matrix(torch.cat([tensors[p + "shared.gate"], tensors[p + "shared.up"]], 0)),
                           runtime.matrix(tensors[p + "shared.down"]), 0.0)      # limit 0: the plain gated unit

    def forward(self, x, batch):
        k = self.runtime.kernels
        choice, weight = k.route_corrected(x, self.w_router, self.correction, self.experts, self.top, self.scale,
                                           NORMALISER_FLOOR)
        # limit 0 and alpha 1: silu(g) * u; the shared expert without a gate of its own
        return k.routed_experts(x, choice, weight, self.w_gate_up, self.w_down, 0.0, 1.0, self.shared, None)   # float32 [T, width]


register_part("feed_forward", "corrected_experts", CorrectedExperts)
