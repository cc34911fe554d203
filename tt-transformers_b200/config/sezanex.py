"""The Sezanex decoder's configuration, read from its own config.json keys.

Top level: `architecture` ("Sezanex"), `vocab`, `width`, `norm.eps`, `layers` and `loop`. A layer gives `type`
("attention": grouped-query softmax attention over a sliding window; "mamba2": a state-space mixer behind a short
causal convolution), `mixer` (its sizes and constants) and `mlp` (a dense or a routed feed-forward, or null).
`loop` {start, stop, times} runs layers start .. stop-1 `times` times in a row. Every size and constant comes from
there; nothing is assumed to be equal between layers.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

from .base import ConfigError, require, take

MIXER_TYPES = ("attention", "mamba2")


@dataclass(frozen=True)
class YarnConfig:
    factor: float
    original: float
    fast: float
    slow: float


@dataclass(frozen=True)
class AttentionConfig:
    heads: int
    kv_heads: int
    dim: int
    vdim: int
    scale: float
    window: Optional[int]
    rot_dims: int
    rot_base: float
    yarn: Optional[YarnConfig]


@dataclass(frozen=True)
class Mamba2Config:
    heads: int
    vdim: int
    state: int
    groups: int
    norm_groups: int
    taps: int


@dataclass(frozen=True)
class MlpConfig:
    kind: str                    # "dense" or "moe"
    inter: int
    experts: int = 0
    top: int = 0


@dataclass(frozen=True)
class SezanexLayer:
    type: str
    mixer: object                # AttentionConfig or Mamba2Config
    mlp: Optional[MlpConfig]


@dataclass(frozen=True)
class SezanexConfig:
    architecture: str
    vocab: int
    width: int
    norm_eps: float
    layers: Tuple[SezanexLayer, ...]
    loop_start: int = 0
    loop_stop: int = 0
    loop_times: int = 0          # 0: no loop (and no matrix at the start of a pass)

    # what the engine's entry points ask of any configuration
    eos_token_ids: tuple = ()
    bos_token_id: Optional[int] = None

    @property
    def vocab_size(self) -> int:
        return self.vocab

    @classmethod
    def from_dict(cls, data: dict) -> "SezanexConfig":
        norm = data.get("norm")
        require(isinstance(norm, dict), "config.json: 'norm' must be an object holding 'eps'")
        raw_layers = data.get("layers")
        require(isinstance(raw_layers, list) and len(raw_layers) >= 1, "config.json: 'layers' must be a non-empty list")
        layers = tuple(_layer(i, entry) for i, entry in enumerate(raw_layers))
        start = stop = times = 0
        loop = data.get("loop")
        if loop is not None:
            require(isinstance(loop, dict), "config.json: 'loop' must be an object or null")
            start, stop = take(loop, "start", int, where="config.json: loop"), take(loop, "stop", int, where="config.json: loop")
            times = take(loop, "times", int, where="config.json: loop")
            require(0 <= start < stop <= len(layers), f"config.json: loop: start {start} .. stop {stop} must name layers of the {len(layers)}")
            require(times >= 1, "config.json: loop: 'times' must be at least 1")
        cfg = cls(architecture=take(data, "architecture", str), vocab=take(data, "vocab", int),
                  width=take(data, "width", int), norm_eps=take(norm, "eps", float, where="config.json: norm"), layers=layers,
                  loop_start=start, loop_stop=stop, loop_times=times)
        require(cfg.vocab >= 1 and cfg.width >= 1, "config.json: 'vocab' and 'width' must be positive")
        return cfg


def _positive(obj, keys, where):
    for key in keys:
        require(getattr(obj, key) >= 1, f"{where}: '{key}' must be positive")


def _attention(m: dict, where: str) -> AttentionConfig:
    rot, mask = m.get("rot"), m.get("mask")
    require(rot is None or isinstance(rot, dict), f"{where}: 'rot' must be an object holding 'base' and 'dims'")
    require(mask is None or isinstance(mask, dict), f"{where}: 'mask' must be an object holding 'size'")
    yarn = None
    scaling = rot.get("scaling") if rot else None
    if scaling is not None:
        w = where + ".rot.scaling"
        require(isinstance(scaling, dict), f"{w} must be an object holding 'factor', 'original', 'fast' and 'slow'")
        yarn = YarnConfig(factor=take(scaling, "factor", float, where=w), original=take(scaling, "original", float, where=w),
                          fast=take(scaling, "fast", float, where=w), slow=take(scaling, "slow", float, where=w))
        require(yarn.factor > 0 and yarn.original > 0 and yarn.fast > 0 and yarn.slow > 0, f"{w}: every value must be positive")
    cfg = AttentionConfig(heads=take(m, "heads", int, where=where), kv_heads=take(m, "kv_heads", int, where=where),
                          dim=take(m, "dim", int, where=where), vdim=take(m, "vdim", int, where=where),
                          scale=take(m, "scale", float, where=where),
                          window=take(mask, "size", int, where=where + ".mask") if mask else None,
                          rot_dims=take(rot, "dims", int, where=where + ".rot") if rot else 0,
                          rot_base=take(rot, "base", float, where=where + ".rot") if rot else 0.0, yarn=yarn)
    _positive(cfg, ("heads", "kv_heads", "dim", "vdim"), where)
    require(cfg.heads % cfg.kv_heads == 0, f"{where}: 'heads' ({cfg.heads}) must be a multiple of 'kv_heads' ({cfg.kv_heads})")
    require(cfg.rot_dims % 2 == 0 and 0 <= cfg.rot_dims <= cfg.dim,
            f"{where}: rot.dims ({cfg.rot_dims}) must be even and at most 'dim' ({cfg.dim})")
    require(cfg.rot_dims == 0 or cfg.rot_base > 0, f"{where}: rot.base must be positive")
    require(cfg.window is None or cfg.window >= 1, f"{where}: mask.size must be positive")
    return cfg


def _mamba2(m: dict, where: str) -> Mamba2Config:
    cfg = Mamba2Config(heads=take(m, "heads", int, where=where), vdim=take(m, "vdim", int, where=where),
                       state=take(m, "state", int, where=where), groups=take(m, "groups", int, where=where),
                       norm_groups=take(m, "norm_groups", int, 1, where=where), taps=take(m, "conv", int, where=where))
    _positive(cfg, ("heads", "vdim", "state", "groups", "norm_groups", "taps"), where)
    require(cfg.heads % cfg.groups == 0, f"{where}: 'heads' ({cfg.heads}) must be a multiple of 'groups' ({cfg.groups})")
    require((cfg.heads * cfg.vdim) % cfg.norm_groups == 0,
            f"{where}: heads * vdim ({cfg.heads * cfg.vdim}) must split into 'norm_groups' ({cfg.norm_groups}) equal parts")
    return cfg


def _mlp(raw, where: str) -> Optional[MlpConfig]:
    if raw is None:
        return None
    require(isinstance(raw, dict), f"{where} must be an object or null")
    kind = take(raw, "kind", str, where=where)
    if kind == "dense":
        cfg = MlpConfig(kind=kind, inter=take(raw, "ff", int, where=where))
        require(cfg.inter >= 1, f"{where}: 'ff' must be positive")
        return cfg
    if kind != "moe":
        raise ConfigError(f"{where}: kind {kind!r} is not known; known: ['dense', 'moe']")
    expert, router = raw.get("expert"), raw.get("router")
    require(isinstance(expert, dict) and isinstance(router, dict), f"{where}: 'expert' and 'router' must be objects")
    cfg = MlpConfig(kind=kind, inter=take(expert, "ff", int, where=where + ".expert"),
                    experts=take(router, "experts", int, where=where + ".router"),
                    top=take(router, "top", int, where=where + ".router"))
    require(cfg.inter >= 1, f"{where}.expert: 'ff' must be positive")
    require(1 <= cfg.top <= cfg.experts, f"{where}.router: 'top' must lie between 1 and 'experts'")
    return cfg


def _layer(i: int, entry) -> SezanexLayer:
    where = f"config.json: layers[{i}]"
    require(isinstance(entry, dict), f"{where} must be an object")
    kind = take(entry, "type", str, where=where)
    require(kind in MIXER_TYPES, f"{where}: type {kind!r} is not known; known: {list(MIXER_TYPES)}")
    m = entry.get("mixer")
    require(isinstance(m, dict), f"{where}: 'mixer' must be an object")
    mixer = _attention(m, where + ".mixer") if kind == "attention" else _mamba2(m, where + ".mixer")
    return SezanexLayer(type=kind, mixer=mixer, mlp=_mlp(entry.get("mlp"), where + ".mlp"))
