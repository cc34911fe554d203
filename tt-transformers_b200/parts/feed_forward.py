"""SwiGLU feed-forward: (silu(x W1) * (x W3)) W2, no biases.

src/tt_transformers/modules/mlp/mlp_1d.py:240-294; tests/modules/mlp/test_mlp_1d.py:676.
Gate (W1) and up (W3) are stacked into one matrix so that one product reads x once.
"""

from __future__ import annotations

import torch

from .base import FeedForward, TensorSpec, register_part


class SwiGLU(FeedForward):
    graph_safe = True

    def __init__(self, width: int, inter: int, prefix: str):
        self.width, self.inter, self.prefix = int(width), int(inter), prefix

    def tensor_specs(self):
        p = self.prefix
        return [TensorSpec(p + "gate_proj.weight", (self.inter, self.width)),
                TensorSpec(p + "up_proj.weight", (self.inter, self.width)),
                TensorSpec(p + "down_proj.weight", (self.width, self.inter))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        self.w_gate_up = runtime.matrix(torch.cat([tensors[p + "gate_proj.weight"], tensors[p + "up_proj.weight"]], 0))
        self.w_down = runtime.matrix(tensors[p + "down_proj.weight"])

    fuses_norm = True
    fuses_residual = True

    def forward(self, x, batch, residual=None, next_norm=None):
        k = self.runtime.kernels
        h = k.linear_swiglu(x, self.w_gate_up)
        if residual is not None:
            # ADDED or a DeferredNorm where the product's epilogue takes the add, else the product itself
            return k.linear(h, self.w_down, accumulate=residual, next_norm=next_norm)
        return k.linear(h, self.w_down)


register_part("feed_forward", "swiglu", SwiGLU)


class GatedMLP(FeedForward):
    """W_down (act(W_gate h) * (W_up h)) with the activation and the tensor names as parameters: `activation`
    "silu", "relu" or "gelu_tanh" (0.5 z (1 + tanh(sqrt(2/pi) (z + 0.044715 z^3)))); `names` = (gate, up, down) after
    `prefix`. The activation is computed in float32 on the product's output."""

    graph_safe = True

    def __init__(self, width: int, inter: int, prefix: str, activation: str = "silu", names=("gate", "up", "down")):
        self.width, self.inter, self.prefix, self.activation = int(width), int(inter), prefix, activation
        self.names = tuple(names)
        if activation not in ("silu", "gelu_tanh", "relu"):
            raise ValueError(f"activation {activation!r} is not known; known: ['silu', 'gelu_tanh', 'relu']")

    def tensor_specs(self):
        p, (g, u, d) = self.prefix, self.names
        return [TensorSpec(p + g, (self.inter, self.width)), TensorSpec(p + u, (self.inter, self.width)),
                TensorSpec(p + d, (self.width, self.inter))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p, (g, u, d) = self.prefix, self.names
        self.w_gate_up = runtime.matrix(torch.cat([tensors[p + g], tensors[p + u]], 0))
        self.w_down = runtime.matrix(tensors[p + d])

    def forward(self, x, batch):
        k = self.runtime.kernels
        if self.activation == "silu":
            return k.linear(k.linear_swiglu(x, self.w_gate_up), self.w_down)
        return k.linear(k.glu_activation(k.linear(x, self.w_gate_up), self.activation), self.w_down)


register_part("feed_forward", "gated_mlp", GatedMLP)


class PlainMLP(FeedForward):
    """W_down act(W_up h) without a gate; `activation` "gelu_erf" (0.5 z (1 + erf(z / sqrt 2))); `names` = (up, down)
    after `prefix`. The activation is computed in float32 on the product's output."""

    graph_safe = True

    def __init__(self, width: int, inter: int, prefix: str, activation: str = "gelu_erf", names=("up", "down")):
        self.width, self.inter, self.prefix, self.activation = int(width), int(inter), prefix, activation
        self.names = tuple(names)
        if activation not in ("gelu_erf",):
            raise ValueError(f"activation {activation!r} is not known; known: ['gelu_erf']")

    def tensor_specs(self):
        p, (u, d) = self.prefix, self.names
        return [TensorSpec(p + u, (self.inter, self.width)), TensorSpec(p + d, (self.width, self.inter))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p, (u, d) = self.prefix, self.names
        self.w_up = runtime.matrix(tensors[p + u])
        self.w_down = runtime.matrix(tensors[p + d])

    def forward(self, x, batch):
        k = self.runtime.kernels
        return k.linear(k.activation(k.linear(x, self.w_up), self.activation, x.dtype), self.w_down)


register_part("feed_forward", "mlp", PlainMLP)
