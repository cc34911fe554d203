"""How norm, mixer and feed-forward are arranged in one layer.

`pre_norm`: h = norm(x); x = x + mixer(h); h = norm(x); x = x + ff(h)
(src/tt_transformers/models/llama32_1b/model.py:113-139,141-186). The residual stream x
is float32. A sub-layer's output is not added at once: it is handed on as `delta` and
added inside the next norm kernel, which reads and writes x once instead of twice.

Parts that say so fuse further: a sub-layer with `fuses_residual` is given the stream and the norm
that follows, and may add its output to the stream itself (its last product's epilogue does it)
and prepare that norm on the way (ADDED or a DeferredNorm comes back); a norm with `can_defer`
before a sub-layer with `fuses_norm` hands the DeferredNorm on, and that sub-layer's first product
finishes it. A decode layer then runs no norm kernel at all. Parts without these flags see
tensors only, as before.
"""

from __future__ import annotations

from .base import ADDED, Block, DeferredNorm, PendingDelta, ScaledParts, SumDelta, register_part


def _normed(norm, consumer, x, delta):
    if getattr(norm, "can_defer", False):
        return norm.forward_add(x, delta, defer=bool(getattr(consumer, "fuses_norm", False)))
    if delta is ADDED or isinstance(delta, DeferredNorm):
        delta = None                             # the stream is up to date; this norm knows tensors only
    return norm.forward_add(x, delta)


def _following(norm, consumer):
    """The norm to prepare in a sub-layer's last product: only one that can take it, before a part that can."""
    if norm is not None and getattr(norm, "can_defer", False) and getattr(consumer, "fuses_norm", False):
        return norm
    return None


class PreNormBlock(Block):
    slots = {"norm1": "norm", "mixer": "mixer", "norm2": "norm", "feed_forward": "feed_forward"}
    takes_next_norm = True

    def __init__(self, norm1, mixer, norm2, feed_forward):
        self.norm1, self.mixer, self.norm2, self.feed_forward = norm1, mixer, norm2, feed_forward

    def forward(self, x, delta, batch, cache, write_cache=True, next_norm=None):
        """x: float32 residual, updated in place; delta: pending sub-layer output, None, or ADDED
        (nothing pending) or a DeferredNorm made for norm1. next_norm: the norm that the caller will
        run on the result, if what follows it can take a DeferredNorm. Returns (x, delta)."""
        h = _normed(self.norm1, self.mixer, x, delta)
        if getattr(self.mixer, "fuses_residual", False):
            mixed = self.mixer.forward(h, batch, cache, write_cache, residual=x,
                                       next_norm=_following(self.norm2, self.feed_forward))
        else:
            mixed = self.mixer.forward(h, batch, cache, write_cache)
        h = _normed(self.norm2, self.feed_forward, x, mixed)
        if getattr(self.feed_forward, "fuses_residual", False):
            return x, self.feed_forward.forward(h, batch, residual=x, next_norm=next_norm)
        return x, self.feed_forward.forward(h, batch)


register_part("block", "pre_norm", PreNormBlock)


class NormedDelta(PendingDelta):
    """A sub-layer's output that still has to pass a norm of its own and a multiplier before it joins the stream."""

    def __init__(self, tensor, norm, mult):
        self.tensor, self.norm, self.mult = tensor, norm, mult

    def settle(self, residual):
        self.norm.join(residual, self.tensor, self.mult)


class SandwichBlock(Block):
    """A norm before and a norm after each sub-layer, and a multiplier m on what joins the stream:
        x += m * post1(mixer(norm1(x)));  x += m * post2(ff(norm2(x))).
    The stream is float32. A sub-layer's output is not added at once: the kernel of the next norm before a
    sub-layer first runs the pending norm-after, adds, and then norms the sum, reading and writing the stream
    once (the second sub-layer's output travels to the next block, or to the model's end, as a NormedDelta).
    Norm parts need `forward_add(x, delta, after=, mult=)` and `join` (kind `layernorm`)."""

    slots = {"norm1": "norm", "mixer": "mixer", "post1": "norm", "norm2": "norm", "feed_forward": "feed_forward",
             "post2": "norm"}
    takes_pending = True

    def __init__(self, norm1, mixer, post1, norm2=None, feed_forward=None, post2=None, residual_mult: float = 1.0):
        self.norm1, self.mixer, self.post1 = norm1, mixer, post1
        self.norm2, self.feed_forward, self.post2 = norm2, feed_forward, post2
        self.residual_mult = float(residual_mult)

    @staticmethod
    def _normed(norm, x, delta):
        if isinstance(delta, NormedDelta):
            return norm.forward_add(x, delta.tensor, after=delta.norm, mult=delta.mult)
        if isinstance(delta, PendingDelta):
            delta.settle(x)
            delta = None
        return norm.forward_add(x, delta)

    def forward(self, x, delta, batch, cache, write_cache=True):
        h = self._normed(self.norm1, x, delta)
        pending = NormedDelta(self.mixer.forward(h, batch, cache, write_cache), self.post1, self.residual_mult)
        if self.feed_forward is None:
            return x, pending
        h = self._normed(self.norm2, x, pending)
        return x, NormedDelta(self.feed_forward.forward(h, batch), self.post2, self.residual_mult)


class SandwichMixerBlock(SandwichBlock):
    """The same block for a layer without a feed-forward: x += m * post1(mixer(norm1(x)))."""

    slots = {"norm1": "norm", "mixer": "mixer", "post1": "norm"}

    def graph_safe(self) -> bool:
        return bool(getattr(self.mixer, "graph_safe", False))


register_part("block", "sandwich", SandwichBlock)
register_part("block", "sandwich_mixer_only", SandwichMixerBlock)


class ParallelBlock(Block):
    """One norm, and both sub-layers read its output: h = norm1(x); x += m (mixer(h) + ff(h)). The outputs travel
    on as one SumDelta and are added to the float32 stream inside the next norm's kernel (the norm part must take a
    SumDelta: kinds `rmsnorm` and `layernorm`). `residual_mult` is m. A mixer that returns a weighted sum of parts
    (ScaledParts) has its parts added there one by one, each with its factor times m."""

    slots = {"norm1": "norm", "mixer": "mixer", "feed_forward": "feed_forward"}
    takes_pending = True

    def __init__(self, norm1, mixer, feed_forward=None, residual_mult: float = 1.0):
        self.norm1, self.mixer, self.feed_forward = norm1, mixer, feed_forward
        self.residual_mult = float(residual_mult)

    def forward(self, x, delta, batch, cache, write_cache=True):
        if isinstance(delta, PendingDelta) and not isinstance(delta, SumDelta):
            delta.settle(x)
            delta = None
        if delta is ADDED or isinstance(delta, DeferredNorm):
            delta = None
        h = self.norm1.forward_add(x, delta)
        mixed = self.mixer.forward(h, batch, cache, write_cache)
        fed = self.feed_forward.forward(h, batch) if self.feed_forward is not None else None
        m = self.residual_mult
        if not isinstance(mixed, ScaledParts):
            return x, SumDelta([mixed, fed], self.mixer.runtime.kernels, scales=None if m == 1.0 else [m, m])
        terms = list(mixed.terms) + ([(fed, 1.0)] if fed is not None else [])
        row = None if mixed.row_term is None else (mixed.row_term[0], mixed.row_term[1] * m)
        return x, SumDelta([t for t, _ in terms], self.mixer.runtime.kernels, scales=[s * m for _, s in terms], row_term=row)


class ParallelMixerBlock(ParallelBlock):
    """The same block for a layer without a feed-forward: x += mixer(norm1(x))."""

    slots = {"norm1": "norm", "mixer": "mixer"}

    def graph_safe(self) -> bool:
        return bool(getattr(self.mixer, "graph_safe", False))


register_part("block", "parallel", ParallelBlock)
register_part("block", "parallel_mixer_only", ParallelMixerBlock)
