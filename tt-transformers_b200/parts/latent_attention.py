"""Attention over a cached low-rank latent.

Per token the cache holds one vector: the latent c (`kv_rank` numbers, RMS-normed) and, where the mixer has
a rotated part, `rot_dim` more numbers, one rotated key part that all heads share. Keys and values of a
head are linear in c (k = W_uk c, v = W_uv c), so neither is ever materialised: the head's query is carried
into the latent space, q' = W_uk^T q, the scores are q' . c (+ q_rot . k_rot), the weighted sum of the
latents comes back through W_uv. Per step and layer the cache is read once, whatever the number of heads.

    c_q = RMS(W_dq h) * g_q;  q = W_uq c_q  (per head [dim | rot_dim])
    [c_raw | k_rot] = W_dkv h;  c = RMS(c_raw) * g_kv
    score_h(i, j) = (q_h,plain(i) . W_uk,h c(j) + R(i) q_h,rot(i) . R(j) k_rot(j)) * scale,  j <= i
    weights: softmax over j, with exp(sink_h) added to the denominator where the mixer has sinks
    o_h(i) = W_uv,h sum_j weight(i, j) c(j);  out = W_o (o * sigmoid(W_g h))

Options, all parameters: `rot_dim` 0 leaves positions out altogether; `sink` adds one learned number per
head to the softmax's denominator (it has no key and no value and is not scaled); `gate` is "element"
(one gate number per output element of the heads), "head" (one per head) or None; `q_rank` None: the queries
come from one matrix, q = W_q h, without a latent of their own; `window` w: position i sees j > i - w only;
`own_latent` False: the mixer has no W_dkv and reads the rows that an earlier layer wrote (its cache unit belongs
to that layer; `keep_window` of that layer is then the widest window of its readers, so that the pages all of them
need stay). A position encoding with `interleaved` pairs the rotated part's elements 2i and 2i + 1: the rows of the
matrices that produce the rotated parts are reordered once, at load, so that the kernels' pairs (i, i + dims/2) are
those; a dot product does not care in which order its terms come. The encoding's amplitude multiplies cosines and
sines of both sides. Norms, rotation angles, scores and softmax are float32. The down projections of one input (W_dq,
W_dkv, W_g) run as one product.
"""

from __future__ import annotations

from typing import Optional

import torch

from .base import LatentPages, Mixer, PositionEncoding, TensorSpec, register_part


class LatentAttention(Mixer):
    graph_safe = True

    def __init__(self, width: int, heads: int, dim: int, vdim: int, q_rank: Optional[int], kv_rank: int, scale: float,
                 eps: float, prefix: str, rot_dim: int = 0, sink: bool = False, gate: Optional[str] = None,
                 position: Optional[PositionEncoding] = None, window: Optional[int] = None, own_latent: bool = True,
                 keep_window="same"):
        self.width, self.heads, self.dim, self.vdim = int(width), int(heads), int(dim), int(vdim)
        self.q_rank, self.kv_rank, self.rot_dim = (None if q_rank is None else int(q_rank)), int(kv_rank), int(rot_dim)
        self.scale, self.eps, self.prefix = float(scale), float(eps), prefix
        self.sink, self.gate, self.position = bool(sink), gate, position
        self.window = None if window is None else int(window)
        self.own_latent = bool(own_latent)
        self.keep_window = self.window if keep_window == "same" else keep_window      # what the cache keeps readable
        if gate not in (None, "element", "head"):
            raise ValueError(f"gate must be 'element', 'head' or None, got {gate!r}")
        if self.rot_dim and (position is None or not hasattr(position, "rotary_dim")):
            raise ValueError("a mixer with a rotated part needs a rotary position encoding")
        if self.window is not None and self.window < 1:
            raise ValueError("window must be positive")
        if self.keep_window is not None and self.window is not None and self.keep_window < self.window:
            raise ValueError("the cache must keep at least the mixer's own window")
        if self.keep_window is not None and self.window is None:
            raise ValueError("a mixer that sees every position needs a cache that keeps every position")
        if self.rot_dim and position.rotary_dim > self.rot_dim:
            raise ValueError(f"the rotation covers {position.rotary_dim} elements, the rotated part has {self.rot_dim}")

    @property
    def gate_rows(self) -> int:
        return {None: 0, "element": self.heads * self.vdim, "head": self.heads}[self.gate]

    def tensor_specs(self):
        p, H = self.prefix, self.heads
        if self.q_rank is None:
            specs = [TensorSpec(p + "q", (H * (self.dim + self.rot_dim), self.width))]
        else:
            specs = [TensorSpec(p + "dq", (self.q_rank, self.width)), TensorSpec(p + "dq.norm", (self.q_rank,)),
                     TensorSpec(p + "uq", (H * (self.dim + self.rot_dim), self.q_rank))]
        if self.own_latent:
            specs += [TensorSpec(p + "dkv", (self.kv_rank + self.rot_dim, self.width)),
                      TensorSpec(p + "dkv.norm", (self.kv_rank,))]
        specs += [TensorSpec(p + "uk", (H * self.dim, self.kv_rank)), TensorSpec(p + "uv", (H * self.vdim, self.kv_rank)),
                  TensorSpec(p + "o", (self.width, H * self.vdim))]
        if self.sink:
            specs.append(TensorSpec(p + "sink", (H,)))
        if self.gate:
            specs.append(TensorSpec(p + "g", (self.gate_rows, self.width)))
        return specs

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        p, H = self.prefix, self.heads
        rotary_dim = self.position.rotary_dim if self.rot_dim else 0
        pairs_apart = None
        if self.rot_dim and getattr(self.position, "interleaved", False):
            # neighbours (2i, 2i + 1) of the first rotary_dim elements go to (i, i + rotary_dim/2)
            pairs_apart = torch.cat([torch.arange(0, rotary_dim, 2), torch.arange(1, rotary_dim, 2),
                                     torch.arange(rotary_dim, self.rot_dim)])

        def rotated_rows_apart(w, first, rows_per_unit, units):
            """w's rows come in `units` runs of rows_per_unit; in each, the rotated part starts at row `first`."""
            if pairs_apart is None:
                return w
            w = w.clone().view(units, rows_per_unit, -1)
            w[:, first:first + self.rot_dim] = w[:, first:first + self.rot_dim][:, pairs_apart]
            return w.view(units * rows_per_unit, -1)

        down = []
        if self.q_rank is not None:
            down.append(tensors[p + "dq"])
        if self.own_latent:
            down.append(rotated_rows_apart(tensors[p + "dkv"], self.kv_rank, self.kv_rank + self.rot_dim, 1))
        if self.gate:
            down.append(tensors[p + "g"])
        self.w_down = runtime.matrix(torch.cat(down, 0)) if down else None   # [q_rank + kv_rank + rot_dim + gate rows, width]
        self.w_uq = runtime.matrix(rotated_rows_apart(tensors[p + ("uq" if self.q_rank is not None else "q")], self.dim,
                                                      self.dim + self.rot_dim, H))
        # per head, the matrix that carries a query into the latent space: (W_uk,h)^T as [kv_rank, dim]
        self.w_uk_t = runtime.matrix(tensors[p + "uk"].view(H, self.dim, self.kv_rank).transpose(1, 2))
        self.w_uv = runtime.matrix(tensors[p + "uv"].view(H, self.vdim, self.kv_rank))
        self.w_o = runtime.matrix(tensors[p + "o"])
        f32 = dict(device=runtime.device, dtype=torch.float32)
        self.q_norm = tensors[p + "dq.norm"].to(**f32).contiguous() if self.q_rank is not None else None
        self.kv_norm = tensors[p + "dkv.norm"].to(**f32).contiguous() if self.own_latent else None
        self.amplitude = float(getattr(self.position, "amplitude", 1.0)) if self.rot_dim else 1.0
        self.sinks = tensors[p + "sink"].to(**f32).contiguous() if self.sink else None

    def cache_request(self):
        return LatentPages(self.kv_rank, self.rot_dim, self.keep_window)

    def forward(self, x, batch, cache, write_cache=True):
        k = self.runtime.kernels
        H, D, R, rot = self.heads, self.dim, self.kv_rank, self.rot_dim
        inv_freq, rotary_dim = self.position.rotation() if rot else (None, 0)
        q_rank = self.q_rank or 0
        own = self.own_latent and write_cache
        extra = {} if self.amplitude == 1.0 else {"amplitude": self.amplitude}
        down = c_q = None
        if self.w_down is not None:
            down = k.linear(x, self.w_down, out_dtype=torch.float32)
        if q_rank or own:
            # the query latent, normed; the key/value latent, normed, and the rotated key part into the pages
            c_q = k.latent_prepare(down, batch, q_rank, R, rot, self.q_norm, self.kv_norm, self.eps, inv_freq, rotary_dim,
                                   cache, own, self.runtime.dtype, **extra)
        q = k.linear(c_q if q_rank else x, self.w_uq).view(-1, H, D + rot)
        q_latent = k.heads_linear(q[:, :, :D], self.w_uk_t)                       # [T, H, R]
        gate = down[:, q_rank + (R + rot if self.own_latent else 0):] if self.gate else None
        if self.window is not None:
            extra["window"] = self.window
        # the weighted sums of the latents [T, H, R], through W_uv per head, gated: [T, H * vdim]
        out = k.latent_attention_out(q_latent, q[:, :, D:] if rot else None, batch, cache, self.scale, self.sinks,
                                     inv_freq, rotary_dim, self.w_uv, gate, **extra)
        return k.linear(out, self.w_o)


register_part("mixer", "latent_attention", LatentAttention)
