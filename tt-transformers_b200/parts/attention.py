"""Grouped-query attention over the paged cache.

One fused projection gives queries, keys and values (no bias); queries and keys are
rotated by their positions; keys and values go into the cache pages at their
positions; every query then attends, causally, to the keys of its request that the
cache holds, the ones just written included; the heads are concatenated and projected.
Order of operations: src/tt_transformers/modules/attention/attention_1d.py:507-518
(projection), :557-571 (rotation of q and k), :576-601 (cache write), :650-659 (causal
attention, scale head_dim^-0.5 :1641-1642), :699-706 (output projection).
Weights stay in the checkpoint's [out, in] layout and the checkpoint's row order, on
which the rotation pairs element i with i + head_dim/2.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import Mixer, PagedKV, PositionEncoding, TensorSpec, register_part


class Attention(Mixer):
    graph_safe = True

    def __init__(self, width: int, heads: int, kv_heads: int, head_dim: int, prefix: str,
                 position: Optional[PositionEncoding] = None, scale: Optional[float] = None,
                 window: Optional[int] = None):
        if heads % kv_heads:
            raise ValueError(f"heads ({heads}) must be a multiple of kv_heads ({kv_heads})")
        self.width, self.heads, self.kv_heads, self.head_dim = int(width), int(heads), int(kv_heads), int(head_dim)
        self.prefix, self.position, self.window = prefix, position, window
        self.scale = float(scale) if scale is not None else self.head_dim ** -0.5
        if position is not None and getattr(position, "amplitude", 1.0) != 1.0:
            raise ValueError("this mixer's kernels rotate with amplitude 1; the position encoding asks for another one")

    def tensor_specs(self):
        q, kv = self.heads * self.head_dim, self.kv_heads * self.head_dim
        return [TensorSpec(self.prefix + "q_proj.weight", (q, self.width)),
                TensorSpec(self.prefix + "k_proj.weight", (kv, self.width)),
                TensorSpec(self.prefix + "v_proj.weight", (kv, self.width)),
                TensorSpec(self.prefix + "o_proj.weight", (self.width, q))]

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        fused = torch.cat([tensors[p + "q_proj.weight"], tensors[p + "k_proj.weight"], tensors[p + "v_proj.weight"]], 0)
        self.w_qkv = runtime.matrix(fused)
        self.w_o = runtime.matrix(tensors[p + "o_proj.weight"])

    def cache_request(self):
        return PagedKV(self.kv_heads, self.head_dim, self.window)

    fuses_norm = True
    fuses_residual = True

    def step_tables_signature(self):
        return ("attention", self.heads // self.kv_heads)

    def step_tables(self, seg_lens, seg_pos0, fixed_tokens=0):
        """The query-tile lists that the attention kernels want for this step, as host tables: they travel with
        the step's metadata in its one copy to the device and reach forward() in batch.extras."""
        return self.runtime.kernels.attention_tables(seg_lens, seg_pos0, self.heads // self.kv_heads, fixed_tokens)

    def forward(self, x, batch, cache, write_cache=True, residual=None, next_norm=None):
        k = self.runtime.kernels
        rotation = self.position.rotation() if self.position is not None else None
        inv_freq, rotary_dim = rotation if rotation is not None else (None, 0)
        interleaved = bool(getattr(self.position, "interleaved", False))
        qkv = None
        if batch.max_seg_len == 1:          # a handful of decoded tokens: projection, rotation and cache write in one kernel
            qkv = k.fused_qkv_rope(x, self.w_qkv, batch, inv_freq, rotary_dim, self.heads, self.kv_heads, self.head_dim,
                                   cache, write_cache, interleaved=interleaved)
        if qkv is None:
            qkv = k.linear(x, self.w_qkv)
            k.rope_kv_write(qkv, batch, inv_freq, rotary_dim, self.heads, self.kv_heads, self.head_dim, cache, write_cache,
                            interleaved=interleaved)
        mixed = k.paged_attention(qkv, batch, self.heads, self.kv_heads, self.head_dim, self.scale, cache)
        if residual is not None:
            # ADDED or a DeferredNorm where the product's epilogue takes the add, else the product itself
            return k.linear(mixed, self.w_o, accumulate=residual, next_norm=next_norm)
        return k.linear(mixed, self.w_o)


register_part("mixer", "attention", Attention)
