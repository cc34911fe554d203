"""Two mixers side by side: both read the same input. `combine` "rms_mean": each output is RMS-normed over the
model width with a plain weight of its own, and the result is their mean:

    out = (rms(left(h)) * w_left + rms(right(h)) * w_right) / 2

`combine` "weighted": out = left_scale * left(h) + right_scale * right(h), with factors from the configuration and no
tensors of the pair's own. The sum is not formed here: the parts come back as ScaledParts, and the block adds them to the
stream with their factors in the kernel of its next norm (a mixer's output bias travels as the row term).

The two mixers are parts of any registered kind, given as PartSpecs; each keeps what it asks of the cache
(the layer's cache unit is a tuple of theirs). The layer's position encoding goes to the mixers named in
`positioned`.
"""

from __future__ import annotations

import torch

from .base import Mixer, PartSpec, ScaledParts, TensorSpec, build_part, register_part


class MixerPair(Mixer):
    def __init__(self, width: int, eps: float, left: PartSpec, right: PartSpec, left_norm: str = None, right_norm: str = None,
                 positioned=("left",), position=None, combine: str = "rms_mean", left_scale: float = 1.0,
                 right_scale: float = 1.0):
        self.width, self.eps = int(width), float(eps)
        self.left_norm, self.right_norm = left_norm, right_norm
        self.combine, self.left_scale, self.right_scale = combine, float(left_scale), float(right_scale)
        if combine not in ("rms_mean", "weighted"):
            raise ValueError(f"combine {combine!r} is not known; known: ['rms_mean', 'weighted']")
        if combine == "rms_mean" and (left_norm is None or right_norm is None):
            raise ValueError("combine 'rms_mean' needs the names of the two norm weights")

        def build(name, spec):
            if position is not None and name in positioned:
                spec = PartSpec(spec.kind, dict(spec.params, position=position))
            return build_part("mixer", spec)

        self.left, self.right = build("left", left), build("right", right)
        requests = [m.cache_request() for m in (self.left, self.right)]
        self._requests = requests
        self.graph_safe = bool(getattr(self.left, "graph_safe", False) and getattr(self.right, "graph_safe", False))

    def tensor_specs(self):
        own = [TensorSpec(self.left_norm, (self.width,)), TensorSpec(self.right_norm, (self.width,))] if self.combine == "rms_mean" else []
        return self.left.tensor_specs() + self.right.tensor_specs() + own

    def bind(self, tensors, runtime):
        super().bind(tensors, runtime)
        self.left.bind(tensors, runtime)
        self.right.bind(tensors, runtime)
        f32 = dict(device=runtime.device, dtype=torch.float32)
        if self.combine == "rms_mean":
            self.w_left = tensors[self.left_norm].to(**f32).contiguous()
            self.w_right = tensors[self.right_norm].to(**f32).contiguous()
        # both mixers project the same input: where both say which rows they need, one product serves them
        self.w_both = None
        if all(hasattr(m, "input_weight") for m in (self.left, self.right)):
            a, b = self.left.input_weight, self.right.input_weight
            if a.dtype == b.dtype and a.shape[1] == b.shape[1] and a.shape[0] % 8 == 0:
                self.w_both = torch.cat([a, b], 0).contiguous()
                self.rows_left = a.shape[0]
                self.left.input_weight = self.w_both[:self.rows_left]          # the same storage, not a second copy
                self.right.input_weight = self.w_both[self.rows_left:]

    def cache_request(self):
        kept = tuple(r for r in self._requests if r is not None)
        return kept or None

    def step_tables_signature(self):
        return ("pair",) + tuple(m.step_tables_signature() if hasattr(m, "step_tables_signature") else id(m)
                                 for m in (self.left, self.right))

    def step_tables(self, seg_lens, seg_pos0, fixed_tokens=0):
        tables = {}
        for m in (self.left, self.right):
            if hasattr(m, "step_tables"):
                tables.update(m.step_tables(seg_lens, seg_pos0, fixed_tokens))
        return tables

    def forward(self, x, batch, cache, write_cache=True):
        views = iter(cache or ())
        outs = []
        slices = (None, None)
        if self.w_both is not None:
            both = self.runtime.kernels.linear(x, self.w_both)
            slices = (both[:, :self.rows_left], both[:, self.rows_left:])
        weighted = self.combine == "weighted"
        row_term = None
        for m, request, projected, scale in zip((self.left, self.right), self._requests, slices, (self.left_scale, self.right_scale)):
            view = next(views) if request is not None else None
            kwargs = {} if projected is None else {"projected": projected}
            if weighted and getattr(m, "output_bias", None) is not None:
                if row_term is not None:
                    raise ValueError("one output bias per pair travels as the row term")
                kwargs["add_output_bias"] = False
                row_term = (m.output_bias, scale)
            outs.append(m.forward(x, batch, view, write_cache, **kwargs))
        if weighted:
            return ScaledParts([(outs[0], self.left_scale), (outs[1], self.right_scale)], row_term, self.runtime.kernels)
        return self.runtime.kernels.mean_rmsnorm_pair(outs[0], self.w_left, outs[1], self.w_right, self.eps)


register_part("mixer", "mixer_pair", MixerPair)
