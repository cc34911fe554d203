"""The Bufolorn decoder's configuration, read from its own config.json keys.

Top level: `architecture` ("Bufolorn"), `vocab`, `width`, `norm.eps`, `embedding.scale`, `residual_mult` and `layers`.
A layer gives `type` ("channel_delta": a delta rule with a decay per key channel behind short convolutions;
"parallel": softmax attention with a learned distance bias beside a decayed outer-product state with token shift;
"latent_attention": attention over a cached latent with a sliding window, optionally reading another layer's latent
through `kv_from`), `mixer` (its sizes and constants) and `mlp` (a dense or a routed feed-forward, or null). Every size
and constant comes from there; nothing is assumed to be equal between layers. Ranks of the low-rank maps are read from
the tensors' shapes by the loader; the optional keys `decay_rank`, `gate_rank` and `bias_rows` give them where tensors
are made up instead of read (random models).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

from .base import ConfigError, require, take

MIXER_TYPES = ("channel_delta", "parallel", "latent_attention")


@dataclass(frozen=True)
class DeltaConfig:
    heads: int
    kv_heads: int
    dim: int
    vdim: int
    taps: int
    decay_rank: Optional[int] = None     # ranks of the low-rank maps: None reads them from the checkpoint's shapes
    gate_rank: Optional[int] = None


@dataclass(frozen=True)
class BiasedAttentionConfig:
    heads: int
    kv_heads: int
    dim: int
    vdim: int
    scale: float
    softcap: Optional[float]
    bias_max: int
    temp_coef: float             # 0: no query temperature
    temp_every: int
    bias_rows: Optional[int] = None      # rows of the distance table: None reads them from the checkpoint


@dataclass(frozen=True)
class ShiftedStateConfig:
    heads: int
    dim: int
    decay_rank: Optional[int] = None


@dataclass(frozen=True)
class SideBySideConfig:
    left: BiasedAttentionConfig
    right: ShiftedStateConfig
    left_scale: float
    right_scale: float


@dataclass(frozen=True)
class BlendConfig:
    factor: float
    original: float
    fast: float
    slow: float


@dataclass(frozen=True)
class LatentConfig:
    heads: int
    dim: int
    rot_dim: int
    vdim: int
    kv_rank: int
    scale: float
    window: Optional[int]
    rot_dims: int
    rot_base: float
    blend: Optional[BlendConfig]
    kv_from: Optional[int]


@dataclass(frozen=True)
class MlpConfig:
    kind: str                    # "dense" or "moe"
    inter: int
    experts: int = 0
    top: int = 0
    router_scale: float = 1.0
    shared_inter: Optional[int] = None


@dataclass(frozen=True)
class BufolornLayer:
    type: str
    mixer: object                # DeltaConfig, SideBySideConfig or LatentConfig
    mlp: Optional[MlpConfig]


@dataclass(frozen=True)
class BufolornConfig:
    architecture: str
    vocab: int
    width: int
    norm_eps: float
    embedding_scale: float
    residual_mult: float
    layers: Tuple[BufolornLayer, ...]

    # what the engine's entry points ask of any configuration
    eos_token_ids: tuple = ()
    bos_token_id: Optional[int] = None

    @property
    def vocab_size(self) -> int:
        return self.vocab

    @classmethod
    def from_dict(cls, data: dict) -> "BufolornConfig":
        norm = data.get("norm")
        require(isinstance(norm, dict), "config.json: 'norm' must be an object holding 'eps'")
        emb = data.get("embedding") or {}
        require(isinstance(emb, dict), "config.json: 'embedding' must be an object")
        raw_layers = data.get("layers")
        require(isinstance(raw_layers, list) and len(raw_layers) >= 1, "config.json: 'layers' must be a non-empty list")
        layers = tuple(_layer(i, entry) for i, entry in enumerate(raw_layers))
        for i, layer in enumerate(layers):
            m = layer.mixer
            if isinstance(m, LatentConfig) and m.kv_from is not None:
                where = f"config.json: layers[{i}].mixer"
                require(0 <= m.kv_from < i, f"{where}: 'kv_from' ({m.kv_from}) must name an earlier layer")
                src = layers[m.kv_from].mixer
                require(isinstance(src, LatentConfig) and src.kv_from is None,
                        f"{where}: 'kv_from' ({m.kv_from}) must name a latent_attention layer with a latent of its own")
                require((src.kv_rank, src.rot_dim, src.rot_dims, src.rot_base, src.blend) ==
                        (m.kv_rank, m.rot_dim, m.rot_dims, m.rot_base, m.blend),
                        f"{where}: 'kv_rank', 'rot_dim' and 'rot' must equal those of layer {m.kv_from}, whose latent it reads")
        cfg = cls(architecture=take(data, "architecture", str), vocab=take(data, "vocab", int),
                  width=take(data, "width", int), norm_eps=take(norm, "eps", float, where="config.json: norm"),
                  embedding_scale=take(emb, "scale", float, 1.0, where="config.json: embedding"),
                  residual_mult=take(data, "residual_mult", float, 1.0), layers=layers)
        require(cfg.vocab >= 1 and cfg.width >= 1, "config.json: 'vocab' and 'width' must be positive")
        return cfg


def _positive(obj, keys, where):
    for key in keys:
        require(getattr(obj, key) >= 1, f"{where}: '{key}' must be positive")


def _delta(m: dict, where: str) -> DeltaConfig:
    cfg = DeltaConfig(heads=take(m, "heads", int, where=where), kv_heads=take(m, "kv_heads", int, where=where),
                      dim=take(m, "dim", int, where=where), vdim=take(m, "vdim", int, where=where),
                      taps=take(m, "conv", int, where=where), decay_rank=take(m, "decay_rank", int, None, where=where),
                      gate_rank=take(m, "gate_rank", int, None, where=where))
    _positive(cfg, ("heads", "kv_heads", "dim", "vdim", "taps"), where)
    require(cfg.heads % cfg.kv_heads == 0, f"{where}: 'heads' ({cfg.heads}) must be a multiple of 'kv_heads' ({cfg.kv_heads})")
    return cfg


def _biased_attention(m: dict, where: str) -> BiasedAttentionConfig:
    temp = m.get("q_temp")
    require(temp is None or isinstance(temp, dict), f"{where}: 'q_temp' must be an object holding 'coef' and 'every'")
    cfg = BiasedAttentionConfig(
        heads=take(m, "heads", int, where=where), kv_heads=take(m, "kv_heads", int, where=where),
        dim=take(m, "dim", int, where=where), vdim=take(m, "vdim", int, where=where),
        scale=take(m, "scale", float, where=where), softcap=take(m, "softcap", float, None, where=where),
        bias_max=take(m, "bias_max", int, where=where),
        temp_coef=take(temp, "coef", float, where=where + ".q_temp") if temp else 0.0,
        temp_every=take(temp, "every", int, where=where + ".q_temp") if temp else 1,
        bias_rows=take(m, "bias_rows", int, None, where=where))
    _positive(cfg, ("heads", "kv_heads", "dim", "vdim", "bias_max", "temp_every"), where)
    require(cfg.heads % cfg.kv_heads == 0, f"{where}: 'heads' ({cfg.heads}) must be a multiple of 'kv_heads' ({cfg.kv_heads})")
    require(cfg.softcap is None or cfg.softcap > 0, f"{where}: 'softcap' must be positive")
    return cfg


def _shifted_state(m: dict, where: str) -> ShiftedStateConfig:
    cfg = ShiftedStateConfig(heads=take(m, "heads", int, where=where), dim=take(m, "dim", int, where=where),
                             decay_rank=take(m, "decay_rank", int, None, where=where))
    _positive(cfg, ("heads", "dim"), where)
    return cfg


def _latent(m: dict, where: str) -> LatentConfig:
    rot, mask = m.get("rot"), m.get("mask")
    require(rot is None or isinstance(rot, dict), f"{where}: 'rot' must be an object holding 'base' and 'dims'")
    require(mask is None or isinstance(mask, dict), f"{where}: 'mask' must be an object holding 'size'")
    blend = None
    if rot and rot.get("scaling") is not None:
        sc = rot["scaling"]
        require(isinstance(sc, dict), f"{where}.rot: 'scaling' must be an object")
        w = where + ".rot.scaling"
        blend = BlendConfig(factor=take(sc, "factor", float, where=w), original=take(sc, "original", float, where=w),
                            fast=take(sc, "fast", float, where=w), slow=take(sc, "slow", float, where=w))
        require(blend.factor > 0 and blend.original > 0 and blend.fast > 0 and blend.slow > 0, f"{w}: every value must be positive")
    cfg = LatentConfig(
        heads=take(m, "heads", int, where=where), dim=take(m, "dim", int, where=where),
        rot_dim=take(m, "rot_dim", int, 0, where=where), vdim=take(m, "vdim", int, where=where),
        kv_rank=take(m, "kv_rank", int, where=where), scale=take(m, "scale", float, where=where),
        window=take(mask, "size", int, where=where + ".mask") if mask else None,
        rot_dims=take(rot, "dims", int, where=where + ".rot") if rot else 0,
        rot_base=take(rot, "base", float, where=where + ".rot") if rot else 0.0, blend=blend,
        kv_from=take(m, "kv_from", int, None, where=where))
    _positive(cfg, ("heads", "dim", "vdim", "kv_rank"), where)
    require(cfg.rot_dim >= 0 and cfg.rot_dims % 2 == 0 and 0 <= cfg.rot_dims <= cfg.rot_dim,
            f"{where}: rot.dims ({cfg.rot_dims}) must be even and at most 'rot_dim' ({cfg.rot_dim})")
    require(cfg.rot_dims == 0 or cfg.rot_base > 0, f"{where}.rot: 'base' must be positive")
    require(cfg.window is None or cfg.window >= 1, f"{where}: mask.size must be positive")
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
    expert, router, shared = raw.get("expert"), raw.get("router"), raw.get("shared")
    require(isinstance(expert, dict) and isinstance(router, dict), f"{where}: 'expert' and 'router' must be objects")
    require(shared is None or isinstance(shared, dict), f"{where}: 'shared' must be an object or null")
    cfg = MlpConfig(kind=kind, inter=take(expert, "ff", int, where=where + ".expert"),
                    experts=take(router, "experts", int, where=where + ".router"),
                    top=take(router, "top", int, where=where + ".router"),
                    router_scale=take(router, "scale", float, 1.0, where=where + ".router"),
                    shared_inter=take(shared, "ff", int, where=where + ".shared") if shared else None)
    require(cfg.inter >= 1, f"{where}.expert: 'ff' must be positive")
    require(1 <= cfg.top <= cfg.experts, f"{where}.router: 'top' must lie between 1 and 'experts'")
    require(cfg.shared_inter is None or cfg.shared_inter >= 1, f"{where}.shared: 'ff' must be positive")
    return cfg


def _layer(i: int, entry) -> BufolornLayer:
    where = f"config.json: layers[{i}]"
    require(isinstance(entry, dict), f"{where} must be an object")
    kind = take(entry, "type", str, where=where)
    require(kind in MIXER_TYPES, f"{where}: type {kind!r} is not known; known: {list(MIXER_TYPES)}")
    m = entry.get("mixer")
    require(isinstance(m, dict), f"{where}: 'mixer' must be an object")
    if kind == "channel_delta":
        mixer = _delta(m, where + ".mixer")
    elif kind == "latent_attention":
        mixer = _latent(m, where + ".mixer")
    else:
        left, right = m.get("left"), m.get("right")
        require(isinstance(left, dict) and isinstance(right, dict), f"{where}.mixer: 'left' and 'right' must be objects")
        mixer = SideBySideConfig(left=_biased_attention(left, where + ".mixer.left"),
                                 right=_shifted_state(right, where + ".mixer.right"),
                                 left_scale=take(m, "left_scale", float, 1.0, where=where + ".mixer"),
                                 right_scale=take(m, "right_scale", float, 1.0, where=where + ".mixer"))
    return BufolornLayer(type=kind, mixer=mixer, mlp=_mlp(entry.get("mlp"), where + ".mlp"))
