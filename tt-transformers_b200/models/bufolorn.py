"""The Bufolorn decoder as a ModelSpec.

A scaled embedding table; per layer a `parallel` block (one layer norm with a bias whose output feeds both the mixer
and the feed-forward; both outputs join the float32 stream together, times the residual multiplier) around one of
three mixers: `delta_rule` (type "channel_delta"), a `mixer_pair` with `combine="weighted"` of `sink_attention`
(biases, a weightless per-head norm of queries and keys, a query temperature, a cap, a learned distance bias, a
sink per head, no rotation) and `shifted_state` (type "parallel"), or `latent_attention` without a query latent,
with a sliding window and a rotation of neighbouring pairs with blended frequencies (type "latent_attention"); a
layer with `kv_from` reads the cache unit of the layer it names and has no down projection of its own. The
feed-forward is a `gated_mlp` with relu or `corrected_experts`. A final layer norm and an untied linear head.
Tensor names: 'embed', 'l<i>.norm1' (+ '.b'), 'l<i>.mix.*', 'l<i>.mlp.*', 'final.norm' (+ '.b'), 'head'.
"""

from __future__ import annotations

from ..config.bufolorn import BufolornConfig, DeltaConfig, LatentConfig
from ..parts import LayerCall, LayerSpec, ModelSpec, PartSpec


def load_config(data: dict) -> BufolornConfig:
    return BufolornConfig.from_dict(data)


def _norm(cfg: BufolornConfig, name: str) -> PartSpec:
    return PartSpec("layernorm", dict(width=cfg.width, eps=cfg.norm_eps, weight_name=name, bias_name=name + ".b"))


def _feed_forward(cfg: BufolornConfig, f, prefix: str) -> PartSpec:
    if f.kind == "dense":
        return PartSpec("gated_mlp", dict(width=cfg.width, inter=f.inter, prefix=prefix, activation="relu",
                                          names=("gate", "up", "down")))
    return PartSpec("corrected_experts", dict(width=cfg.width, experts=f.experts, top=f.top, inter=f.inter, prefix=prefix,
                                              scale=f.router_scale, shared_inter=f.shared_inter))


def _kept_window(cfg: BufolornConfig, owner: int):
    """What the latent cache of layer `owner` must keep readable: the widest window among the layer itself and the
    layers that read its latent; None (everything) if one of them sees every position."""
    windows = [cfg.layers[owner].mixer.window]
    windows += [l.mixer.window for l in cfg.layers if isinstance(l.mixer, LatentConfig) and l.mixer.kv_from == owner]
    return None if any(w is None for w in windows) else max(windows)


def model_spec(cfg: BufolornConfig) -> ModelSpec:
    layers, order = [], []
    for i, layer in enumerate(cfg.layers):
        p, m = f"l{i}.", layer.mixer
        position, cache_of = None, None
        if isinstance(m, DeltaConfig):
            mixer = PartSpec("delta_rule", dict(width=cfg.width, heads=m.heads, kv_heads=m.kv_heads, dim=m.dim, vdim=m.vdim,
                                                taps=m.taps, eps=cfg.norm_eps, prefix=p + "mix.",
                                                decay_rank=m.decay_rank, gate_rank=m.gate_rank))
        elif isinstance(m, LatentConfig):
            owner = i if m.kv_from is None else m.kv_from
            cache_of = m.kv_from
            mixer = PartSpec("latent_attention", dict(
                width=cfg.width, heads=m.heads, dim=m.dim, vdim=m.vdim, q_rank=None, kv_rank=m.kv_rank, scale=m.scale,
                eps=cfg.norm_eps, prefix=p + "mix.", rot_dim=m.rot_dim, window=m.window, own_latent=m.kv_from is None,
                keep_window=_kept_window(cfg, owner)))
            if m.rot_dim:
                scaling = None
                if m.blend is not None:
                    b = m.blend
                    scaling = {"type": "blend", "factor": b.factor, "original": b.original, "fast": b.fast, "slow": b.slow}
                position = PartSpec("rotary", dict(rotary_dim=m.rot_dims, theta=m.rot_base, scaling=scaling, interleaved=True))
        else:
            a, r = m.left, m.right
            left = PartSpec("sink_attention", dict(
                width=cfg.width, heads=a.heads, kv_heads=a.kv_heads, dim=a.dim, vdim=a.vdim, scale=a.scale, eps=cfg.norm_eps,
                prefix=p + "mix.left.", softcap=a.softcap, sink=True, qk_norm="plain", bias=True,
                q_temp=(a.temp_coef, a.temp_every), distance_bias=a.bias_max, bias_rows=a.bias_rows))
            right = PartSpec("shifted_state", dict(width=cfg.width, heads=r.heads, dim=r.dim, eps=cfg.norm_eps,
                                                   prefix=p + "mix.right.", decay_rank=r.decay_rank))
            mixer = PartSpec("mixer_pair", dict(width=cfg.width, eps=cfg.norm_eps, left=left, right=right, combine="weighted",
                                                left_scale=m.left_scale, right_scale=m.right_scale, positioned=()))
        parts = dict(norm1=_norm(cfg, p + "norm1"), mixer=mixer)
        params = dict(residual_mult=cfg.residual_mult)
        if layer.mlp is None:
            layers.append(LayerSpec(block="parallel_mixer_only", position=position, block_params=params, **parts))
        else:
            layers.append(LayerSpec(block="parallel", position=position, block_params=params,
                                    feed_forward=_feed_forward(cfg, layer.mlp, p + "mlp."), **parts))
        order.append(LayerCall(i, cache_of=cache_of))
    return ModelSpec(
        vocab_size=cfg.vocab, width=cfg.width,
        embedding=PartSpec("table", dict(vocab=cfg.vocab, width=cfg.width, weight_name="embed", scale=cfg.embedding_scale)),
        layers=tuple(layers), order=tuple(order),
        final_norm=_norm(cfg, "final.norm"),
        head=PartSpec("linear", dict(vocab=cfg.vocab, width=cfg.width, weight_name="head")),
    )


def ignorable(cfg: BufolornConfig, name: str) -> bool:
    return False
