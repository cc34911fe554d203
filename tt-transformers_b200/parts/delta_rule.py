"""A delta-rule mixer with a decay per key channel and a matrix state per head.

    q, k = W_q h, W_k h  [kv_heads, dim];  v = W_v h  [heads, vdim];  each passes a causal convolution per channel
    (`taps` taps, no bias, zeros before the start) and silu; head h reads q and k of head floor(h / (heads / kv_heads))
    q, k <- x / sqrt(sum(x^2) + 1e-6) per head;  q <- q * dim^(-1/2)
    beta = sigmoid(W_b h)  [heads];   g = exp(-exp(A_log_h) softplus(W_a2 (W_a1 h) + dt_bias))  [heads, dim]
    S <- diag(g) S;   u = beta (v - S^T k);   S <- S + k u^T;   o = S^T q          (S: dim x vdim, float32)
    out = W_o (rms_head(o) * g_norm * sigmoid(W_g2 (W_g1 h)))                        (g_norm: vdim numbers, shared by the heads)

The state and the convolutions' last taps - 1 inputs live in a slot per live request, zero at the start. The unit
norms, beta, the decay's map behind its first product with its softplus and exponentials, the recurrence, the head
norm and the gate are float32; the projections and the convolutions with their silu leave in the compute dtype.
`decay_rank`, `gate_rank` None read the ranks of the two low-rank maps from the checkpoint.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import MatrixState, Mixer, TensorSpec, register_part

UNIT_FLOOR = 1e-6       # inside the root of the unit norm


class DeltaRule(Mixer):
    graph_safe = True

    def __init__(self, width: int, heads: int, kv_heads: int, dim: int, vdim: int, taps: int, eps: float, prefix: str,
                 decay_rank: Optional[int] = None, gate_rank: Optional[int] = None, position=None):
        self.width, self.heads, self.kv_heads, self.dim, self.vdim = int(width), int(heads), int(kv_heads), int(dim), int(vdim)
        self.taps, self.eps, self.prefix = int(taps), float(eps), prefix
        self.decay_rank = None if decay_rank is None else int(decay_rank)
        self.gate_rank = None if gate_rank is None else int(gate_rank)
        if self.heads % self.kv_heads:
            raise ValueError(f"heads ({heads}) must be a multiple of kv_heads ({kv_heads})")
        if self.taps < 1:
            raise ValueError("the convolution needs at least one tap")
        self.qk, self.inner = self.kv_heads * self.dim, self.heads * self.vdim
        self.channels = 2 * self.qk + self.inner              # what the convolutions run over: q, k, v

    def tensor_specs(self):
        p, H = self.prefix, self.heads
        return [TensorSpec(p + "q", (self.qk, self.width)), TensorSpec(p + "q.conv", (self.qk, self.taps)),
                TensorSpec(p + "k", (self.qk, self.width)), TensorSpec(p + "k.conv", (self.qk, self.taps)),
                TensorSpec(p + "v", (self.inner, self.width)), TensorSpec(p + "v.conv", (self.inner, self.taps)),
                TensorSpec(p + "b", (H, self.width)), TensorSpec(p + "A_log", (H,)), TensorSpec(p + "norm", (self.vdim,)),
                TensorSpec(p + "a1", (self.decay_rank, self.width)), TensorSpec(p + "a2", (H * self.dim, self.decay_rank)),
                TensorSpec(p + "dt_bias", (H * self.dim,)),
                TensorSpec(p + "g1", (self.gate_rank, self.width)), TensorSpec(p + "g2", (self.inner, self.gate_rank)),
                TensorSpec(p + "o", (self.width, self.inner))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        f32 = dict(device=runtime.device, dtype=torch.float32)
        self.w_qkv = runtime.matrix(torch.cat([tensors[p + "q"], tensors[p + "k"], tensors[p + "v"]], 0))
        self.conv = torch.cat([tensors[p + "q.conv"], tensors[p + "k.conv"], tensors[p + "v.conv"]], 0).to(**f32).contiguous()
        # beta's rows and the first halves of the two low-rank maps: one small product, float32 out
        self.w_small = runtime.matrix(torch.cat([tensors[p + "b"], tensors[p + "a1"], tensors[p + "g1"]], 0))
        self.ranks = (tensors[p + "a1"].shape[0], tensors[p + "g1"].shape[0])
        self.w_a2 = runtime.matrix(tensors[p + "a2"])
        self.w_g2 = runtime.matrix(tensors[p + "g2"])
        self.dt_bias = tensors[p + "dt_bias"].to(**f32).contiguous()
        # exp(A_log) does not depend on the token: once, in float32
        self.rate = torch.exp(tensors[p + "A_log"].to(torch.float32)).to(**f32).contiguous()
        self.norm = tensors[p + "norm"].to(**f32).contiguous()
        self.w_o = runtime.matrix(tensors[p + "o"])

    def cache_request(self):
        return MatrixState(self.heads, self.dim, self.vdim, self.channels, self.taps)

    def forward(self, x, batch, cache, write_cache=True):
        k = self.runtime.kernels
        H, (ra, rg) = self.heads, self.ranks
        qkv = k.linear(x, self.w_qkv)                                             # [T, q | k | v] before the convolutions
        small = k.linear(x, self.w_small, out_dtype=torch.float32)                # [T, beta | a1 | g1]
        u = k.short_conv_silu(qkv, self.conv, batch, cache)                       # [T, q | k | v]
        log_decay = k.lowrank_expand(small[:, H:H + ra], self.w_a2, self.dt_bias, None, "neg_rate_softplus",
                                     rate=self.rate)                              # float32 [T, heads * dim] = ln g
        gate = k.lowrank_expand(small[:, H + ra:H + ra + rg], self.w_g2, None, None, "none")       # float32 [T, heads * vdim]
        mixed = k.delta_rule(u, qkv, small[:, :H], log_decay, gate, self.norm, self.eps, self.heads, self.kv_heads, self.dim,
                             self.vdim, batch, cache, write_cache)
        return k.linear(mixed, self.w_o)


register_part("mixer", "delta_rule", DeltaRule)
