"""A recurrent mixer with token shift and a decayed outer-product state per head (the time mixing of Peng et al.,
"RWKV: Reinventing RNNs for the Transformer Era", 2023, with a decay that depends on the token).

    h' = the token before (zeros before the first);  mix_s = h + (h' - h) * mu_s        for s in r, k, v, g, w
    r, k, v = W_r mix_r, W_k mix_k, W_v mix_v  [heads, dim];   gate = silu(W_g mix_g)
    w = exp(-exp(W_w2 tanh(W_w1 mix_w) + w0))                                           [heads, dim], one per key channel
    o_t = (S_(t-1) + diag(u) k_t v_t^T)^T r_t;    S_t = diag(w_t) S_(t-1) + k_t v_t^T     (u: a bonus for the current token)
    out = W_o (rms_head(o) * g_norm * gate)

The state S [heads, dim, dim] (float32) and the previous token's input live in a slot per live request, zero at the
start. The mixes, the decay's low-rank map behind its first product, its exponentials, the recurrence, the head norm
and the gate are float32; the five mixes are rounded to the compute dtype for their products. `decay_rank` None reads
the rank of the decay's map from the checkpoint.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import MatrixState, Mixer, TensorSpec, register_part

MIXES = ("r", "k", "v", "g", "w")


class ShiftedState(Mixer):
    graph_safe = True
    SKINNY_ROWS = 16        # up to this many tokens the four projections run one by one

    def __init__(self, width: int, heads: int, dim: int, eps: float, prefix: str, decay_rank: Optional[int] = None,
                 position=None):
        self.width, self.heads, self.dim, self.eps, self.prefix = int(width), int(heads), int(dim), float(eps), prefix
        self.decay_rank = None if decay_rank is None else int(decay_rank)
        self.inner = self.heads * self.dim

    def tensor_specs(self):
        p, n = self.prefix, self.inner
        specs = [TensorSpec(p + "mu." + s, (self.width,)) for s in MIXES]
        specs += [TensorSpec(p + s, (n, self.width)) for s in ("r", "k", "v", "g")]
        specs += [TensorSpec(p + "w1", (self.decay_rank, self.width)), TensorSpec(p + "w2", (n, self.decay_rank)),
                  TensorSpec(p + "w0", (n,)), TensorSpec(p + "u", (self.heads, self.dim)), TensorSpec(p + "norm", (n,)),
                  TensorSpec(p + "o", (self.width, n))]
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        f32 = dict(device=runtime.device, dtype=torch.float32)
        self.mu = torch.stack([tensors[p + "mu." + s] for s in MIXES]).to(**f32).contiguous()          # [5, width]
        self.w_rkvg = runtime.matrix(torch.stack([tensors[p + s] for s in ("r", "k", "v", "g")]))       # [4, inner, width]
        self.w_1 = runtime.matrix(tensors[p + "w1"])
        self.w_2 = runtime.matrix(tensors[p + "w2"])
        self.w_0 = tensors[p + "w0"].to(**f32).contiguous()
        self.bonus = tensors[p + "u"].to(**f32).contiguous()
        self.norm = tensors[p + "norm"].to(**f32).contiguous()
        self.w_o = runtime.matrix(tensors[p + "o"])

    def cache_request(self):
        return MatrixState(self.heads, self.dim, self.dim, self.width, 2)      # the state, and one kept input: h'

    def forward(self, x, batch, cache, write_cache=True):
        k = self.runtime.kernels
        mixes = k.token_shift(x, self.mu, batch, cache)                                      # [T, 5, width]
        if x.shape[0] <= self.SKINNY_ROWS:
            # a handful of tokens: four products that stream their weights, each by the kernel made for few rows
            rkvg = [k.linear(mixes[:, i], self.w_rkvg[i]) for i in range(4)]
        else:
            rkvg = k.heads_linear(mixes[:, :4], self.w_rkvg)                                 # [T, 4, inner]
        low = k.linear(mixes[:, 4], self.w_1, out_dtype=torch.float32)                       # [T, rank]
        log_decay = k.lowrank_expand(low, self.w_2, self.w_0, "tanh", "neg_exp")             # float32 [T, inner] = ln w
        mixed = k.shifted_state(rkvg, log_decay, self.bonus, self.norm, self.eps, self.heads, self.dim, x, batch, cache,
                                write_cache)
        return k.linear(mixed, self.w_o)


register_part("mixer", "shifted_state", ShiftedState)
