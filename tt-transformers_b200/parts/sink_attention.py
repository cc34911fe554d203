"""Grouped-query attention with the options of recent decoders, each a parameter:

    q, k, v = W_q h, W_k h, W_v h           (query/key size `dim`, value size `vdim`, no biases)
    qk_norm:   True or "head": q and k are RMS-normed per head over `dim` with one weight each, shared by the heads;
               "whole": the RMS norm runs over the whole of q (all heads at once) and over the whole of k, with a
               weight per element of the projection; before rotation either way
    position:  the first rotary_dim elements of q and k are rotated by the token's position (pairs i, i + rotary_dim/2),
               cosines and sines times the encoding's amplitude
    score = (q . k) * scale;  softcap c: score = c tanh(score / c)
    chunk n:   position i sees j <= i with floor(i / n) = floor(j / n) only;  window w: j > i - w
    sink:      one learned number per head joins the softmax's denominator as exp(sink_h); it has no value;
    sink_score: the same with one constant for every head and no tensor (0: a one in the denominator)
    bias:      q, k, v and the output projection have biases ('<tensor>.b'), added to the products
    qk_norm "plain": the per-head RMS norm without a weight
    q_temp (c, n): the normed query at position p is multiplied by 1 + c ln(floor((p + 1) / n) + 1)
    distance_bias far: a learned table '<prefix>rel' [rows, heads] adds rel[bucket(i - j), h] to the capped score (the
               scale does not touch it); with half = rows // 2: bucket(n) = n below half, else
               min(rows - 1, half + floor(ln(n / half) / ln(far / half) * (rows - half))): single positions near by,
               logarithmic steps up to `far`, one row for everything beyond. The table per distance is laid out once,
               at load, in float64 logarithms.
    out = W_o (heads' weighted sums of v)

Keys (normed, rotated) and values go into cache pages at their positions; pages wholly before a request's
current chunk or window are given back by the cache manager. Norms, angles, scores and softmax are float32.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from .base import Mixer, PagedKV, PositionEncoding, TensorSpec, register_part


class SinkAttention(Mixer):
    graph_safe = True

    def __init__(self, width: int, heads: int, kv_heads: int, dim: int, vdim: int, scale: float, eps: float, prefix: str,
                 softcap: Optional[float] = None, chunk: Optional[int] = None, window: Optional[int] = None,
                 sink: bool = False, qk_norm=False, position: Optional[PositionEncoding] = None,
                 sink_score: Optional[float] = None, bias: bool = False, q_temp=None, distance_bias: Optional[int] = None,
                 bias_rows: Optional[int] = None):
        if heads % kv_heads:
            raise ValueError(f"heads ({heads}) must be a multiple of kv_heads ({kv_heads})")
        self.width, self.heads, self.kv_heads, self.dim, self.vdim = int(width), int(heads), int(kv_heads), int(dim), int(vdim)
        self.scale, self.eps, self.prefix = float(scale), float(eps), prefix
        self.softcap = None if softcap is None else float(softcap)
        self.chunk = None if chunk is None else int(chunk)
        self.window = None if window is None else int(window)
        if qk_norm not in (False, True, None, "head", "whole", "plain"):
            raise ValueError(f"qk_norm {qk_norm!r} is not known; known: [False, 'head', 'whole', 'plain']")
        self.sink, self.qk_norm, self.position = bool(sink), bool(qk_norm), position
        self.whole_norm, self.plain_norm = qk_norm == "whole", qk_norm == "plain"
        self.bias = bool(bias)
        self.q_temp = None if not q_temp or not float(q_temp[0]) else (float(q_temp[0]), int(q_temp[1]))
        self.distance_bias = None if distance_bias is None else int(distance_bias)
        self.bias_rows = bias_rows                   # None: the table's rows are read from the checkpoint
        if self.q_temp is not None and self.q_temp[1] < 1:
            raise ValueError("q_temp: positions are counted in runs of at least one")
        if self.distance_bias is not None and self.distance_bias < 1:
            raise ValueError("distance_bias must be positive")
        self.sink_score = None if sink_score is None else float(sink_score)
        if self.sink and self.sink_score is not None:
            raise ValueError("a learned sink and a constant one exclude each other")
        if self.softcap is not None and not self.softcap > 0:
            raise ValueError("softcap must be positive")
        if self.chunk is not None and self.chunk < 1:
            raise ValueError("chunk must be positive")
        if (self.bias or self.q_temp is not None) and (self.whole_norm or (position is not None and getattr(position, "amplitude", 1.0) != 1.0)):
            raise ValueError("biases and a query temperature come with the per-head norm and rotations of amplitude 1")
        if position is not None and getattr(position, "interleaved", False):
            raise ValueError("neighbouring rotation pairs are not built for this mixer")
        if position is not None and getattr(position, "rotary_dim", 0) > self.dim:
            raise ValueError(f"the rotation covers {position.rotary_dim} elements, a head has {self.dim}")

    def tensor_specs(self):
        p, H, G = self.prefix, self.heads, self.kv_heads
        specs = [TensorSpec(p + "q", (H * self.dim, self.width)), TensorSpec(p + "k", (G * self.dim, self.width)),
                 TensorSpec(p + "v", (G * self.vdim, self.width)), TensorSpec(p + "o", (self.width, H * self.vdim))]
        if self.whole_norm:
            specs += [TensorSpec(p + "q.norm", (H * self.dim,)), TensorSpec(p + "k.norm", (G * self.dim,))]
        elif self.qk_norm and not self.plain_norm:
            specs += [TensorSpec(p + "q.norm", (self.dim,)), TensorSpec(p + "k.norm", (self.dim,))]
        if self.sink:
            specs.append(TensorSpec(p + "sink", (H,)))
        if self.bias:
            specs += [TensorSpec(p + "q.b", (H * self.dim,)), TensorSpec(p + "k.b", (G * self.dim,)),
                      TensorSpec(p + "v.b", (G * self.vdim,)), TensorSpec(p + "o.b", (self.width,))]
        if self.distance_bias is not None:
            specs.append(TensorSpec(p + "rel", (self.bias_rows, H), free_size=16))
        return specs

    @staticmethod
    def distance_bucket(n: int, rows: int, far: int) -> int:
        half = rows // 2
        if n < half or half == 0:
            return min(n, rows - 1)
        if far <= half:
            return rows - 1
        return min(rows - 1, half + int(math.floor(math.log(n / half) / math.log(far / half) * (rows - half))))

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p = self.prefix
        self.w_qkv = runtime.matrix(torch.cat([tensors[p + "q"], tensors[p + "k"], tensors[p + "v"]], 0))
        self.w_o = runtime.matrix(tensors[p + "o"])
        f32 = dict(device=runtime.device, dtype=torch.float32)
        if self.plain_norm:
            self.q_norm = self.k_norm = torch.ones(self.dim, **f32)
        else:
            self.q_norm = tensors[p + "q.norm"].to(**f32).contiguous() if self.qk_norm else None
            self.k_norm = tensors[p + "k.norm"].to(**f32).contiguous() if self.qk_norm else None
        self.b_qkv = self.output_bias = self.bias_by_distance = None
        if self.bias:
            self.b_qkv = torch.cat([tensors[p + "q.b"], tensors[p + "k.b"], tensors[p + "v.b"]], 0).to(**f32).contiguous()
            self.output_bias = tensors[p + "o.b"].to(**f32).contiguous()
        if self.distance_bias is not None:
            # [heads, far + 1]: the bias of every distance up to `far`, beyond which the last row holds
            rel = tensors[p + "rel"].to(torch.float32)
            far = self.distance_bias
            rows = [self.distance_bucket(n, rel.shape[0], far) for n in range(far + 1)]
            self.bias_by_distance = rel[torch.tensor(rows)].t().to(**f32).contiguous()
        self.sinks = tensors[p + "sink"].to(**f32).contiguous() if self.sink else None
        if self.sink_score is not None:
            self.sinks = torch.full((self.heads,), self.sink_score, **f32)
        self.amplitude = float(getattr(self.position, "amplitude", 1.0)) if self.position is not None else 1.0

    def cache_request(self):
        return PagedKV(self.kv_heads, self.dim, self.window, value_dim=self.vdim, chunk=self.chunk)

    def step_tables_signature(self):
        return ("attention", self.heads // self.kv_heads)

    def step_tables(self, seg_lens, seg_pos0, fixed_tokens=0):
        """The query-tile lists that the tensor-core attention kernels want for this step (they travel with the
        step's metadata in its one copy to the device)."""
        return self.runtime.kernels.attention_tables(seg_lens, seg_pos0, self.heads // self.kv_heads, fixed_tokens)

    # a mixer that stands beside another one may get its input projection as a slice of one product for both:
    # `input_weight` is what that product needs of this mixer, `projected` what comes back
    @property
    def input_weight(self):
        return self.w_qkv

    @input_weight.setter
    def input_weight(self, rows):
        self.w_qkv = rows

    def forward(self, x, batch, cache, write_cache=True, projected=None, add_output_bias=True):
        """add_output_bias False: the caller adds `output_bias` itself (on the way into the stream, say)."""
        k = self.runtime.kernels
        rotation = self.position.rotation() if self.position is not None else None
        inv_freq, rotary_dim = rotation if rotation is not None else (None, 0)
        qkv = projected if projected is not None else k.linear(x, self.w_qkv)
        extra = {}
        if self.b_qkv is not None:
            extra["bias"] = self.b_qkv
        if self.q_temp is not None:
            extra["q_temp"] = self.q_temp
        if extra:
            k.qk_norm_rope_write(qkv, batch, self.q_norm, self.k_norm, self.eps, inv_freq, rotary_dim, self.heads,
                                 self.kv_heads, self.dim, self.vdim, cache, write_cache, **extra)
        elif self.whole_norm or self.amplitude != 1.0:
            k.qk_norm_rope_write(qkv, batch, self.q_norm, self.k_norm, self.eps, inv_freq, rotary_dim, self.heads,
                                 self.kv_heads, self.dim, self.vdim, cache, write_cache, whole=self.whole_norm,
                                 amplitude=self.amplitude)
        else:
            k.qk_norm_rope_write(qkv, batch, self.q_norm, self.k_norm, self.eps, inv_freq, rotary_dim, self.heads,
                                 self.kv_heads, self.dim, self.vdim, cache, write_cache)
        extra = {} if self.bias_by_distance is None else {"distance_bias": self.bias_by_distance}
        mixed = k.sink_attention(qkv, batch, self.heads, self.kv_heads, self.dim, self.vdim, self.scale, self.softcap,
                                 self.sinks, cache, **extra)
        out = k.linear(mixed, self.w_o)
        if self.output_bias is not None and add_output_bias:
            k.add_row_vector(out, self.output_bias)
        return out


register_part("mixer", "sink_attention", SinkAttention)
