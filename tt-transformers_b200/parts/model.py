"""A decoder model as data, and the generic model that runs it.

`ModelSpec` names the parts of every layer (kind + parameters), the order in which
layers run, and the embedding, final norm and head. `DecoderModel` builds the parts
from the registries and runs a step. An architecture is a function from its typed
configuration to a ModelSpec; nothing here knows any architecture.

The layer order is a list of `LayerCall`s. A call names the layer to run; by default
it owns a cache unit of its own. `cache_of=j` makes it read (never write) the unit of
the j-th call instead. A layer may be named by several calls (shared weights).
"""

from __future__ import annotations

from dataclasses import dataclass, replace
from typing import Dict, List, Optional

import torch

from .base import ADDED, Block, DeferredNorm, PartSpec, PendingDelta, Runtime, StepBatch, TensorSpec, build_part, block_factory


def _block_graph_safe(block) -> bool:
    safe = getattr(block, "graph_safe", None)
    if callable(safe):
        return bool(safe())
    return all(getattr(p, "graph_safe", False) for p in (block.mixer, block.feed_forward))


class LayerSpec:
    """One layer as data: the block kind, a PartSpec for every part that block kind is built from
    (by the names in its `slots`: norm1, mixer, norm2, feed_forward for `pre_norm`; a block kind with
    more parts, say norms after its sub-layers, names more), and the position encoding handed to
    the layer's mixer as `position`."""

    __slots__ = ("block", "position", "parts", "block_params")

    def __init__(self, block: str = "pre_norm", position: Optional[PartSpec] = None, block_params: Optional[dict] = None,
                 **parts: PartSpec):
        for name, spec in parts.items():
            if not isinstance(spec, PartSpec):
                raise TypeError(f"LayerSpec: part {name!r} must be a PartSpec, got {type(spec).__name__}")
        self.block, self.position, self.parts = block, position, dict(parts)
        self.block_params = dict(block_params or {})     # constants of the block kind itself (a residual multiplier)

    def __getattr__(self, name):                 # spec.mixer, spec.norm1, ... read like fields
        parts = object.__getattribute__(self, "parts")
        if name in parts:
            return parts[name]
        raise AttributeError(name)

    def __repr__(self):
        return f"LayerSpec(block={self.block!r}, position={self.position!r}, parts={self.parts!r})"


@dataclass(frozen=True)
class LayerCall:
    layer: int
    cache_of: Optional[int] = None           # index into the layer order, earlier than this call


@dataclass(frozen=True)
class ModelSpec:
    vocab_size: int
    width: int
    embedding: PartSpec                      # category "embedding"
    layers: tuple                            # of LayerSpec
    order: tuple                             # of LayerCall
    final_norm: PartSpec
    head: PartSpec                           # category "head"
    input_position: Optional[PartSpec] = None  # a position encoding applied to the embedded tokens
    max_positions: int = 1 << 30
    stream_steps: tuple = ()                 # of (index into the layer order, PartSpec of category "stream_step"):
                                             # what happens to the residual stream right before that entry runs

    def first_entries(self, count: int) -> "ModelSpec":
        """The same model cut to the first `count` entries of its layer order (for runs that want fewer
        layers than the checkpoint has). Layers that no remaining entry names are dropped."""
        if not 1 <= count <= len(self.order):
            raise ValueError(f"the layer order has {len(self.order)} entries; cannot keep {count}")
        order = self.order[:count]
        used = sorted({call.layer for call in order})
        renumber = {old: new for new, old in enumerate(used)}
        return replace(self, layers=tuple(self.layers[i] for i in used),
                       order=tuple(LayerCall(renumber[c.layer], c.cache_of) for c in order),
                       stream_steps=tuple((at, spec) for at, spec in self.stream_steps if at < count))


class DecoderModel:
    def __init__(self, spec: ModelSpec):
        self.spec = spec
        self.embedding = build_part("embedding", spec.embedding)
        self.head = build_part("head", spec.head)
        if getattr(self.head, "tied", False):
            self.head.tie(self.embedding)
        self.final_norm = build_part("norm", spec.final_norm)
        self.input_position = build_part("position", spec.input_position) if spec.input_position else None
        self.layers = []
        positions: Dict[PartSpec, object] = {}
        for number, ls in enumerate(spec.layers):
            position = None
            if ls.position is not None:
                if ls.position not in positions:          # layers with the same encoding share one object
                    positions[ls.position] = build_part("position", ls.position)
                position = positions[ls.position]
            factory = block_factory(ls.block)
            slots = getattr(factory, "slots", Block.slots)
            if set(ls.parts) != set(slots):
                raise ValueError(f"layer {number}: block kind {ls.block!r} is built from {sorted(slots)}, "
                                 f"the layer names {sorted(ls.parts)}")
            built = {}
            for name, category in slots.items():
                part_spec = ls.parts[name]
                if category == "mixer" and position is not None:
                    part_spec = PartSpec(part_spec.kind, dict(part_spec.params, position=position))
                built[name] = build_part(category, part_spec)
            self.layers.append(factory(**built, **ls.block_params))
        self.positions = list(positions.values())
        self.stream_steps = {}
        for at, step_spec in spec.stream_steps:
            if not 0 <= at < len(spec.order):
                raise ValueError(f"a stream step is placed before layer-order entry {at}, which does not exist")
            self.stream_steps.setdefault(at, []).append(build_part("stream_step", step_spec))
        self._keeps_embedding = any(getattr(s, "needs_embedding", False) for ss in self.stream_steps.values() for s in ss)
        for i, call in enumerate(spec.order):
            if not 0 <= call.layer < len(self.layers):
                raise ValueError(f"layer order entry {i} names layer {call.layer}, which does not exist")
            if call.cache_of is not None and not (0 <= call.cache_of < i and spec.order[call.cache_of].cache_of is None):
                raise ValueError(f"layer order entry {i}: cache_of must name an earlier entry that owns its cache")

    # ------------------------------------------------------------------ weights
    def all_parts(self):
        parts = [self.embedding, self.head, self.final_norm]
        if self.input_position is not None:
            parts.append(self.input_position)
        parts.extend(self.positions)
        for steps in self.stream_steps.values():
            parts.extend(steps)
        for block in self.layers:
            parts.extend(block.parts())
        return parts

    def tensor_specs(self) -> List[TensorSpec]:
        seen, out = set(), []
        for part in self.all_parts():
            for spec in part.tensor_specs():
                if spec.name not in seen:
                    seen.add(spec.name)
                    out.append(spec)
        return out

    def bind(self, tensors: Dict[str, torch.Tensor], runtime: Runtime) -> None:
        self.runtime = runtime
        for part in self.all_parts():
            part.bind(tensors, runtime)

    def graph_safe(self) -> bool:
        """True if every mixer and feed-forward says that its forward only launches kernels
        on the current stream with shapes fixed by the batch's shape (no host reads, no
        per-step host tables), so that a decode step may be captured and replayed."""
        return all(_block_graph_safe(b) for b in self.layers)

    def step_tables(self, seg_lens, seg_pos0, fixed_tokens: int = 0) -> Dict[object, object]:
        """Host tables that the mixers want for a step of this shape (Mixer.step_tables), each asked once."""
        if not hasattr(self, "_planners"):
            planners = {}
            for block in self.layers:
                for part in block.parts():
                    if hasattr(part, "step_tables"):
                        sign = part.step_tables_signature() if hasattr(part, "step_tables_signature") else id(part)
                        planners.setdefault(sign, part)
            self._planners = list(planners.values())
        tables = {}
        for part in self._planners:
            tables.update(part.step_tables(seg_lens, seg_pos0, fixed_tokens))
        return tables

    # ------------------------------------------------------------------ cache needs
    def cache_requests(self):
        """For every entry of the layer order: what its cache unit must be (PagedKV,
        SlotState or None), or the index of the entry whose unit it reads."""
        out = []
        for call in self.spec.order:
            if call.cache_of is not None:
                out.append(call.cache_of)
            else:
                out.append(self.layers[call.layer].cache_request())
        return out

    # ------------------------------------------------------------------ one step
    def forward(self, batch: StepBatch, cache) -> torch.Tensor:
        """Run the step's tokens; `cache.view(entry, batch)` gives each entry's cache view.
        Returns float32 logits [num_wanted, vocab]."""
        k = self.runtime.kernels
        x = self.embedding.forward(batch.token_ids)
        if self.input_position is not None:
            x = self.input_position.embed(x, batch)
        delta = None
        order = self.spec.order
        embedded = x.clone() if self._keeps_embedding else None
        for i, call in enumerate(order):
            owner = i if call.cache_of is None else call.cache_of
            block = self.layers[call.layer]
            view = cache.view(owner, batch)
            for step in self.stream_steps.get(i, ()):
                if getattr(step, "settles_first", False) and delta is not None:
                    if isinstance(delta, PendingDelta):
                        delta.settle(x)
                    elif not (delta is ADDED or isinstance(delta, DeferredNorm)):
                        k.stream_add_norm(x, [delta])
                    delta = None
                moved = step.forward(x, embedded, batch)  # in place (an addition commutes with a delta that is still
                if moved is not None:                     # to be added), or a new stream
                    x = moved
            if isinstance(delta, PendingDelta) and not getattr(block, "takes_pending", False):
                delta.settle(x)                   # a block kind that does not know it: plain addition first
                delta = None
            if getattr(block, "takes_next_norm", False):
                # the norm that will run on this block's result, if what follows it can take it half done
                if i + 1 < len(order):
                    nxt = self.layers[order[i + 1].layer]
                    norm, consumer = getattr(nxt, "norm1", None), getattr(nxt, "mixer", None)
                else:
                    norm, consumer = self.final_norm, self.head
                    if not batch.wants_every_row:
                        norm = None              # the head sees a selection of the rows
                ok = (norm is not None and getattr(norm, "can_defer", False) and getattr(consumer, "fuses_norm", False))
                x, delta = block.forward(x, delta, batch, view, write_cache=call.cache_of is None,
                                         next_norm=norm if ok else None)
            else:
                if delta is ADDED or isinstance(delta, DeferredNorm):
                    delta = None
                x, delta = block.forward(x, delta, batch, view, write_cache=call.cache_of is None)
        if isinstance(delta, PendingDelta):
            delta.settle(x)
            delta = None
        if batch.num_wanted == 0:
            return torch.empty(0, self.spec.vocab_size, dtype=torch.float32, device=x.device)
        if isinstance(delta, DeferredNorm) and delta.made_for is self.final_norm and batch.wants_every_row:
            return self.head.forward(self.final_norm.forward_add(x, delta, defer=True))
        if delta is ADDED or isinstance(delta, DeferredNorm):
            delta = None
        if not batch.wants_every_row:
            x = k.gather_rows(x, batch.want_rows)
            if delta is not None:
                delta = k.gather_rows(delta, batch.want_rows)
        h = self.final_norm.forward_add(x, delta)
        return self.head.forward(h)
