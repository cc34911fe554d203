"""A state-space mixer with a matrix state per head (Dao and Gu, "Transformers are SSMs: Generalized Models and
Efficient Algorithms Through Structured State Space Duality", 2024).

    [z | x | B | C | dt] = W_in h          (z, x: heads * vdim each; B, C: groups * state each; dt: heads)
    x, B, C together pass a causal convolution per channel (`taps` taps, a bias, zeros before the start) and silu
    dt = softplus(dt + dt_bias);  a = exp(-exp(A_log_h) dt)                       (per head, float32)
    S_t = a S_(t-1) + dt B_t x_t^T   (S: state x vdim, float32);   y_t = S_t^T C_t + D_h x_t
    out = W_o (rms_groups(y * silu(z)) * w_norm)          (the RMS norm in `norm_groups` equal parts, gate first)

Head h reads B and C of group floor(h / (heads / groups)). The state (float32) and the convolution's last
taps - 1 inputs live in a slot per live request, zero at the start. Step sizes, decays, the recurrence, its output,
the gate and the norm are float32; the projections and the convolution with its activation leave in the compute dtype.
"""

from __future__ import annotations

import torch

from .base import MatrixState, Mixer, TensorSpec, register_part


class StateSpace(Mixer):
    graph_safe = True

    def __init__(self, width: int, heads: int, vdim: int, state: int, groups: int, norm_groups: int, taps: int, eps: float,
                 prefix: str, position=None):
        self.width, self.heads, self.vdim, self.state = int(width), int(heads), int(vdim), int(state)
        self.groups, self.norm_groups, self.taps, self.eps, self.prefix = int(groups), int(norm_groups), int(taps), float(eps), prefix
        self.inner = self.heads * self.vdim
        self.channels = self.inner + 2 * self.groups * self.state        # what the convolution runs over: x, B, C
        if self.heads % self.groups:
            raise ValueError(f"heads ({heads}) must be a multiple of groups ({groups})")
        if self.inner % self.norm_groups:
            raise ValueError(f"heads * vdim ({self.inner}) does not split into {norm_groups} equal parts")
        if self.taps < 1:
            raise ValueError("the convolution needs at least one tap")

    def tensor_specs(self):
        p, H = self.prefix, self.heads
        return [TensorSpec(p + "in", (2 * self.inner + 2 * self.groups * self.state + H, self.width)),
                TensorSpec(p + "conv", (self.channels, self.taps)), TensorSpec(p + "conv.b", (self.channels,)),
                TensorSpec(p + "dt_bias", (H,)), TensorSpec(p + "A_log", (H,)), TensorSpec(p + "D", (H,)),
                TensorSpec(p + "norm", (self.inner,)), TensorSpec(p + "o", (self.width, self.inner))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        f32 = dict(device=runtime.device, dtype=torch.float32)
        self.w_in = runtime.matrix(tensors[p + "in"])
        self.conv = tensors[p + "conv"].to(**f32).contiguous()
        self.conv_b = tensors[p + "conv.b"].to(**f32).contiguous()
        self.dt_bias = tensors[p + "dt_bias"].to(**f32).contiguous()
        # exp(A_log) does not depend on the token: once, in float32
        self.rate = torch.exp(tensors[p + "A_log"].to(torch.float32)).to(**f32).contiguous()
        self.skip = tensors[p + "D"].to(**f32).contiguous()
        self.norm = tensors[p + "norm"].to(**f32).contiguous()
        self.w_o = runtime.matrix(tensors[p + "o"])

    def cache_request(self):
        return MatrixState(self.heads, self.state, self.vdim, self.channels, self.taps)

    def forward(self, x, batch, cache, write_cache=True):
        k = self.runtime.kernels
        proj = k.linear(x, self.w_in)                                   # [T, z | x B C | dt]
        mixed = k.state_space(proj, self.conv, self.conv_b, self.dt_bias, self.rate, self.skip, self.norm, self.eps,
                              self.heads, self.vdim, self.state, self.groups, self.norm_groups, batch, cache, write_cache)
        return k.linear(mixed, self.w_o)


register_part("mixer", "state_space", StateSpace)
