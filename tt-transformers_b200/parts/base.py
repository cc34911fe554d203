"""What a part is, what it may ask of the cache, and where parts are registered.

A part (mixer, feed-forward, norm, position encoding, embedding, head) is built
from a kind name and a dictionary of parameters: all of its sizes and constants.
It declares the checkpoint tensors it needs, takes them at `bind`, and then runs
on the tensors of one step. No part knows which model it is in; the reference
builds its modules the same way, from explicit weights and dimensions
(src/tt_transformers/modules/README.md:18-31,40-66).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple

import torch


# ----------------------------------------------------------------------------- tensors a part needs
@dataclass(frozen=True)
class TensorSpec:
    """One checkpoint tensor: its full name, its shape, and whether it holds
    floating-point values ("float") or an integer table ("int"). A size of None is read from
    the checkpoint (the rank of a low-rank map that no configuration key gives); `free_size`
    stands in for it where tensors are made up (random weights)."""

    name: str
    shape: Tuple[int, ...]
    kind: str = "float"
    optional: bool = False
    free_size: int = 16


# ----------------------------------------------------------------------------- what a mixer asks of the cache
class CacheRequest:
    """What one layer-order entry asks of the cache manager. A request says by itself what is stored
    and how a mixer sees it, so the manager knows no kind of request by name:

    `paged` True: storage per token, in pages handed out through a block table per request;
    `storage(page_size)` gives {name: (shape of ONE page, dtype or None for the compute dtype)}, and the
    manager keeps each tensor as [units, pages + 1, *shape] (page 0 is the scratch page). `window`
    None keeps every position; a number lets the manager take back pages that lie wholly more than
    `window` positions behind the request's end.
    `paged` False: storage of fixed size per live request; `storage(page_size)` gives {name: (shape
    of ONE request's state, dtype)}, kept as [units, slots + 1, *shape] and zeroed when a request is
    admitted (the last row belongs to nobody: padded rows of captured steps point there).

    `view(tensors, ...)` wraps one unit's tensors for the mixer. Requests that compare equal share a
    group (one pool, one block table per request). Subclasses are frozen dataclasses."""

    paged = True
    window = None
    chunk = None     # a number: position i reads keys of its own chunk floor(i / chunk) only; pages wholly before
                     # the chunk that holds a request's end are given back

    def storage(self, page_size: int):
        raise NotImplementedError

    def view(self, tensors, **step):
        raise NotImplementedError


@dataclass(frozen=True)
class PagedKV(CacheRequest):
    """Keys and values in pages. `window` None keeps all keys; a number keeps only
    the last `window` positions readable, and pages behind it are given back. `value_dim` None: values are
    as long as keys. `chunk`: keys are read inside the query's own chunk of that many positions only."""

    num_kv_heads: int
    head_dim: int
    window: Optional[int] = None
    value_dim: Optional[int] = None
    chunk: Optional[int] = None
    paged = True

    def storage(self, page_size: int):
        page = (self.num_kv_heads, page_size, self.head_dim)     # one KV head's page is contiguous
        values = (self.num_kv_heads, page_size, self.value_dim or self.head_dim)
        return {"keys": (page, None), "values": (values, None)}

    def view(self, tensors, *, block_table, page_size, **_):
        return PagedKVView(keys=tensors["keys"], values=tensors["values"], block_table=block_table,
                           page_size=page_size, window=self.window, chunk=self.chunk)


@dataclass(frozen=True)
class SlotState(CacheRequest):
    """A tensor of fixed shape per live request, zeroed when the request is admitted. Mixers with a
    running state of their own use this."""

    shape: Tuple[int, ...]
    dtype: torch.dtype = torch.float32
    paged = False

    def storage(self, page_size: int):
        return {"state": (tuple(self.shape), self.dtype)}

    def view(self, tensors, *, slots, slot_list, **_):
        return SlotStateView(state=tensors["state"], slots=slots, slot_list=slot_list)


@dataclass(frozen=True)
class LatentPages(CacheRequest):
    """One vector per token instead of keys and values: `latent` numbers from which a mixer makes every
    head's key and value, followed by `extra` numbers that are kept as they are (a rotated key part that all
    heads share). A page holds page_size such rows, contiguous."""

    latent: int
    extra: int = 0
    window: Optional[int] = None
    paged = True

    def storage(self, page_size: int):
        return {"rows": ((page_size, self.latent + self.extra), None)}

    def view(self, tensors, *, block_table, page_size, **_):
        return LatentPagesView(rows=tensors["rows"], block_table=block_table, page_size=page_size,
                               latent=self.latent, extra=self.extra, window=self.window)


@dataclass
class LatentPagesView:
    rows: torch.Tensor          # [num_pages, page_size, latent + extra]
    block_table: torch.Tensor   # int32 [segments, pages_per_request]
    page_size: int
    latent: int
    extra: int
    window: Optional[int]


@dataclass
class PagedKVView:
    """One cache unit of a paged group as a mixer sees it during a step."""

    keys: torch.Tensor          # [num_pages, kv_heads, page_size, head_dim]
    values: torch.Tensor        # same shape
    block_table: torch.Tensor   # int32 [segments, pages_per_request]; entry i covers positions i*page_size ..
    page_size: int
    window: Optional[int]
    chunk: Optional[int] = None


@dataclass(frozen=True)
class RecurrentState(CacheRequest):
    """What a gated linear recurrence over `channels` channels behind a short causal convolution keeps per live
    request: the recurrence's state (float32) and the convolution's last `taps - 1` inputs (compute dtype).
    Zeroed at admission."""

    channels: int
    taps: int
    paged = False

    def storage(self, page_size: int):
        return {"state": ((self.channels,), torch.float32), "tail": ((max(self.taps - 1, 1), self.channels), None)}

    def view(self, tensors, *, slots, slot_list, **_):
        return RecurrentStateView(state=tensors["state"], tail=tensors["tail"], taps=self.taps, slots=slots,
                                  slot_list=slot_list)


@dataclass
class RecurrentStateView:
    state: torch.Tensor         # float32 [max_slots + 1, channels]
    tail: torch.Tensor          # [max_slots + 1, taps - 1, channels], oldest input first
    taps: int
    slots: torch.Tensor         # int32 [segments] on the device
    slot_list: List[int]


@dataclass(frozen=True)
class MatrixState(CacheRequest):
    """What a mixer with a matrix-valued recurrence behind a short causal convolution keeps per live request: a
    float32 state [heads, rows, cols] and the convolution's last `taps - 1` inputs over `channels` channels (compute
    dtype). Zeroed at admission."""

    heads: int
    rows: int
    cols: int
    channels: int
    taps: int
    paged = False

    def storage(self, page_size: int):
        return {"state": ((self.heads, self.rows, self.cols), torch.float32),
                "tail": ((max(self.taps - 1, 1), self.channels), None)}

    def view(self, tensors, *, slots, slot_list, **_):
        return MatrixStateView(state=tensors["state"], tail=tensors["tail"], taps=self.taps, slots=slots, slot_list=slot_list)


@dataclass
class MatrixStateView:
    state: torch.Tensor         # float32 [max_slots + 1, heads, rows, cols]
    tail: torch.Tensor          # [max_slots + 1, taps - 1, channels], oldest input first
    taps: int
    slots: torch.Tensor         # int32 [segments] on the device
    slot_list: List[int]


@dataclass
class SlotStateView:
    state: torch.Tensor         # [max_slots + 1, *shape]
    slots: torch.Tensor         # int32 [segments] on the device
    slot_list: List[int]        # the same on the host


# ----------------------------------------------------------------------------- what every part is given
@dataclass
class Runtime:
    """Where and how parts compute: the kernel table, the device, the compute dtype."""

    kernels: object
    device: torch.device
    dtype: torch.dtype          # torch.bfloat16 or torch.float32

    def matrix(self, tensor: torch.Tensor) -> torch.Tensor:
        """A matrix operand on the device in the compute dtype."""
        return tensor.to(device=self.device, dtype=self.dtype).contiguous()

    def vector(self, tensor: torch.Tensor) -> torch.Tensor:
        """A small per-channel vector: a tensor stored in 32-bit stays so, others
        take the compute dtype."""
        dtype = torch.float32 if tensor.dtype == torch.float32 else self.dtype
        return tensor.to(device=self.device, dtype=dtype).contiguous()


@dataclass
class StepBatch:
    """The tokens of one step, flat: segment r owns tokens cu_seqlens[r] ..
    cu_seqlens[r+1]. Device tensors are int32; the host lists mirror them."""

    num_tokens: int
    num_segments: int
    token_ids: torch.Tensor       # [T]
    positions: torch.Tensor       # [T] absolute position of each token in its request
    seg_of_token: torch.Tensor    # [T]
    cu_seqlens: torch.Tensor      # [R+1]
    seg_pos0: torch.Tensor        # [R] tokens of the request cached before this step
    seg_slot: torch.Tensor        # [R]
    want_rows: torch.Tensor       # [N] flat token indices whose logits are wanted
    num_wanted: int
    seg_lens: List[int] = field(default_factory=list)
    seg_pos0_list: List[int] = field(default_factory=list)
    seg_slot_list: List[int] = field(default_factory=list)
    max_seg_len: int = 1
    max_context: int = 1          # the largest pos0 + len over the segments
    wants_every_row: bool = False  # want_rows is 0, 1, .. num_tokens-1
    block_tables: Dict[int, torch.Tensor] = field(default_factory=dict)  # group index -> [R, W]
    extras: dict = field(default_factory=dict)   # per-step tables that kernels derive once and reuse in every layer


class DeferredNorm:
    """A norm whose scaling is still to come. The product that ended the sub-layer before it has
    left `xg` = compute-dtype(g * residual) [rows, width], g being the norm's weight, and `ssq`
    [parts, 16] float32, partial sums of residual^2 per row; the norm's output is
    xg / sqrt(sum(ssq) / width + eps). A skinny matrix product takes this in place of the normalised
    tensor (it divides its sums instead of its input); everything else calls materialize().
    `made_for`: the norm part whose weight and eps went in."""

    __slots__ = ("xg", "ssq", "eps", "made_for", "_materialize")

    def __init__(self, xg, ssq, eps, made_for, materialize):
        self.xg, self.ssq, self.eps, self.made_for, self._materialize = xg, ssq, float(eps), made_for, materialize

    @property
    def shape(self):
        return self.xg.shape

    def materialize(self):
        return self._materialize()


class PendingDelta:
    """A sub-layer output that is not in the residual stream yet and needs more than an addition to get
    there (a norm of its own, a multiplier). A block that knows the kind takes it into its first norm's
    kernel; for everything else `settle(residual)` adds it in place."""

    def settle(self, residual) -> None:
        raise NotImplementedError


class SumDelta(PendingDelta):
    """Several sub-layer outputs (any dtype, each [rows, width]) that join the stream together: a norm that knows
    the kind adds them in its own kernel, everything else calls settle(). `scales`: a factor for each tensor (None:
    all one); `row_term`: (float32 vector [width], factor), the same for every row (a bias on its way into the stream)."""

    def __init__(self, tensors, kernels, scales=None, row_term=None):
        keep = [i for i, t in enumerate(tensors) if t is not None]
        self.tensors, self.kernels = [tensors[i] for i in keep], kernels
        self.scales = None if scales is None else [float(scales[i]) for i in keep]
        self.row_term = row_term
        if self.scales is not None and all(s == 1.0 for s in self.scales):
            self.scales = None

    @property
    def plain(self) -> bool:
        return self.scales is None and self.row_term is None

    def settle(self, residual) -> None:
        if self.plain:
            self.kernels.stream_add_norm(residual, self.tensors)
        else:
            self.kernels.add_layernorm_sum(residual, self.tensors, self.scales, self.row_term, None, None)


class ScaledParts:
    """What a mixer made of mixers returns when its result is a weighted sum that the block may as well form on the
    way into the stream: terms [(tensor [rows, width], factor)] and an optional row term (vector, factor).
    materialize() forms the sum as a float32 tensor for a caller that wants one."""

    def __init__(self, terms, row_term, kernels):
        self.terms, self.row_term, self.kernels = terms, row_term, kernels

    def materialize(self):
        first = self.terms[0][0]
        out = torch.zeros(first.shape, dtype=torch.float32, device=first.device)
        self.kernels.add_layernorm_sum(out, [t for t, _ in self.terms], [s for _, s in self.terms], self.row_term, None, None)
        return out


class _Added:
    """What a part returns instead of its output when it has already added that output to the
    residual stream it was given."""

    def __repr__(self):
        return "ADDED"


ADDED = _Added()


class Part:
    """Base of all parts. Two optional capabilities, off unless a part says otherwise:
    `fuses_norm`: forward() accepts a DeferredNorm in place of x; `fuses_residual`: forward()
    accepts residual=<float32 stream> and next_norm=<the norm part that follows, or None>, may add
    its output to the stream itself and then returns ADDED, or a DeferredNorm made for next_norm."""

    fuses_norm = False
    fuses_residual = False

    def tensor_specs(self) -> List[TensorSpec]:
        return []

    def bind(self, tensors: Dict[str, torch.Tensor], runtime: Runtime) -> None:
        self.runtime = runtime


class Mixer(Part):
    """Mixes information between the positions of a request.

    forward(x [T, width], batch, cache, write_cache) -> [T, width].
    `cache` is the view that matches cache_request(): PagedKVView, SlotStateView or
    None; a mixer whose cache_request() is a tuple of requests gets a tuple of views. With write_cache False the unit belongs to an earlier entry of the
    layer order and must only be read.
    """

    def cache_request(self):
        return None

    def forward(self, x, batch: StepBatch, cache, write_cache: bool = True):
        raise NotImplementedError

    # Optional: step_tables(seg_lens, seg_pos0, fixed_tokens=0) -> {key: int32 numpy array}: small tables that the
    # mixer's kernels derive from the step's shape on the host. They are packed into the step's metadata (one copy
    # to the device) and handed back as device tensors in batch.extras[key]. step_tables_signature() -> hashable:
    # mixers with equal signatures want the same tables (asked once per step). A kernel table without
    # `attention_tables` (a stand-in on the CPU) may return {} from it.


class FeedForward(Part):
    """forward(x [T, width], batch) -> [T, width], each token by itself."""

    def forward(self, x, batch: StepBatch):
        raise NotImplementedError


class Norm(Part):
    """forward_add(residual, delta) adds delta (or nothing, if None) into the
    float32 residual stream in place and returns the normalised tensor in the
    compute dtype. delta may be ADDED (nothing left to add). A norm with `can_defer`
    has fusion_args() -> (float32 weight, eps), accepts a DeferredNorm made for it as delta and,
    with defer=True, may hand it on instead of a tensor."""

    can_defer = False

    def forward_add(self, residual, delta):
        raise NotImplementedError


class PositionEncoding(Part):
    """How positions reach the model. `embed` may change the embedded tokens
    (absolute encodings); `rotation()` gives what a mixer needs to rotate queries
    and keys: (inverse frequencies float32 [rotary_dim/2] on the device,
    rotary_dim), or None when nothing is rotated. `interleaved` says which elements
    of a head form a rotated pair: (i, i + rotary_dim/2) when False, (2i, 2i + 1) when True."""

    interleaved = False

    def embed(self, x, batch: StepBatch):
        return x

    def rotation(self):
        return None


class TokenEmbedding(Part):
    """forward(token_ids int32 [T]) -> float32 [T, width], the start of the residual stream. A head that
    is tied to the embedding reads its `table` ([vocab, width], compute dtype) after bind."""

    def forward(self, token_ids):
        raise NotImplementedError


class OutputHead(Part):
    """forward(h [N, width], compute dtype) -> float32 logits [N, vocab]. A head with `tied` True has no
    weight of its own: the model calls tie(embedding) before bind."""

    tied = False

    def tie(self, embedding: TokenEmbedding) -> None:
        raise NotImplementedError

    def forward(self, h):
        raise NotImplementedError


class StreamStep(Part):
    """Something that happens to the residual stream between two entries of the layer order (the start of a
    pass over looped layers, say). forward(x float32 [T, width], embedded float32 [T, width] or None, batch)
    changes x in place, or returns the new stream; `needs_embedding` True asks the model to keep the embedding's
    output for it. `settles_first` True: the step does more than add to the stream, so a sub-layer output that is
    still on its way there must have joined it before the step runs."""

    needs_embedding = False
    settles_first = False

    def forward(self, x, embedded, batch):
        raise NotImplementedError


class Block:
    """How the parts of one layer are arranged. `slots` names the parts a block kind is built from and
    the category each is looked up in; a LayerSpec gives a PartSpec for every name, the model builds
    them and hands them to the block's constructor as keyword arguments. forward(x, delta, batch,
    cache, write_cache) -> (x, delta): x is the float32 residual stream (updated in place), delta a
    sub-layer output that is still to be added (or None). `mixer` is the part whose cache request
    the entry's cache unit serves and that receives the layer's position encoding."""

    slots: Dict[str, str] = {"norm1": "norm", "mixer": "mixer", "norm2": "norm", "feed_forward": "feed_forward"}
    takes_next_norm = False

    def parts(self):
        return [getattr(self, name) for name in self.slots]

    def cache_request(self):
        return self.mixer.cache_request()

    def graph_safe(self) -> bool:
        """True if the forward of every mixer and feed-forward just launches kernels on the current stream,
        with shapes fixed by the batch's shape."""
        return all(getattr(getattr(self, name), "graph_safe", False)
                   for name, category in self.slots.items() if category in ("mixer", "feed_forward"))

    def forward(self, x, delta, batch, cache, write_cache=True):
        raise NotImplementedError


# ----------------------------------------------------------------------------- registries
_REGISTRIES: Dict[str, Dict[str, Callable]] = {
    "mixer": {}, "feed_forward": {}, "norm": {}, "position": {}, "block": {}, "embedding": {}, "head": {},
    "stream_step": {},
}


def register_part(category: str, kind: str, factory: Callable) -> None:
    """Make `factory(**params)` available as `kind` in `category` (mixer,
    feed_forward, norm, position, block, embedding, head, stream_step). Registering a kind again replaces it."""
    if category not in _REGISTRIES:
        raise KeyError(f"unknown part category {category!r}; known: {sorted(_REGISTRIES)}")
    _REGISTRIES[category][kind] = factory


def block_factory(kind: str) -> Callable:
    table = _REGISTRIES["block"]
    if kind not in table:
        raise KeyError(f"no block of kind {kind!r} is registered; known: {sorted(table)}")
    return table[kind]


def build_part(category: str, spec: "PartSpec"):
    table = _REGISTRIES[category]
    if spec.kind not in table:
        raise KeyError(f"no {category} of kind {spec.kind!r} is registered; known: {sorted(table)}")
    return table[spec.kind](**spec.params)


@dataclass(frozen=True)
class PartSpec:
    """A part as data: which kind, and its parameters (sizes, constants, tensor name prefix)."""

    kind: str
    params: dict = field(default_factory=dict)

    def __hash__(self):
        return hash((self.kind, tuple(sorted((k, repr(v)) for k, v in self.params.items()))))
