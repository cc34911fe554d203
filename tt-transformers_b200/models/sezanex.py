"""The Sezanex decoder as a ModelSpec.

A plain embedding table; per layer a `sandwich` block (a Dynamic Tanh norm before and after each sub-layer, the
stream float32) around a `sink_attention` mixer (norms over the whole query and key projections, a rotation with
blended frequencies and an amplitude, a sliding window, a constant sink of score zero) or a `state_space` mixer,
and an `mlp` (erf-GELU, no gate) or `scored_experts` feed-forward; a final norm of the same kind and a head tied to
the embedding table. Looped layers are named several times in the layer order, each call with a cache unit of its
own; a `pass_mix` stream step stands before the first layer of every pass. Tensor names: 'embed', 'loop.in',
'l<i>.norm1' (with '.b' and '.alpha'), 'l<i>.norm1b', 'l<i>.norm2', 'l<i>.norm2b', 'l<i>.mix.*', 'l<i>.mlp.*',
'final.norm'.
"""

from __future__ import annotations

from ..config.sezanex import SezanexConfig
from ..parts import LayerCall, LayerSpec, ModelSpec, PartSpec

SINK_SCORE = 0.0          # the softmax's denominator holds exp(0) = 1 beside the keys' terms


def load_config(data: dict) -> SezanexConfig:
    return SezanexConfig.from_dict(data)


def _norm(cfg: SezanexConfig, name: str, width: int = None) -> PartSpec:
    return PartSpec("dyntanh", dict(width=width or cfg.width, weight_name=name, bias_name=name + ".b", alpha_name=name + ".alpha"))


def _feed_forward(cfg: SezanexConfig, f, prefix: str) -> PartSpec:
    if f.kind == "dense":
        return PartSpec("mlp", dict(width=cfg.width, inter=f.inter, prefix=prefix, activation="gelu_erf", names=("up", "down")))
    return PartSpec("scored_experts", dict(width=cfg.width, experts=f.experts, top=f.top, inter=f.inter, prefix=prefix,
                                           scores="sigmoid"))


def model_spec(cfg: SezanexConfig) -> ModelSpec:
    layers = []
    for i, layer in enumerate(cfg.layers):
        p, m = f"l{i}.", layer.mixer
        position = None
        if layer.type == "attention":
            mixer = PartSpec("sink_attention", dict(
                width=cfg.width, heads=m.heads, kv_heads=m.kv_heads, dim=m.dim, vdim=m.vdim, scale=m.scale, eps=cfg.norm_eps,
                prefix=p + "mix.", window=m.window, sink_score=SINK_SCORE, qk_norm="whole"))
            if m.rot_dims:
                scaling = None
                if m.yarn is not None:
                    scaling = dict(type="blend", factor=m.yarn.factor, original=m.yarn.original, fast=m.yarn.fast, slow=m.yarn.slow)
                position = PartSpec("rotary", dict(rotary_dim=m.rot_dims, theta=m.rot_base, scaling=scaling))
        else:
            mixer = PartSpec("state_space", dict(width=cfg.width, heads=m.heads, vdim=m.vdim, state=m.state, groups=m.groups,
                                                 norm_groups=m.norm_groups, taps=m.taps, eps=cfg.norm_eps, prefix=p + "mix."))
        parts = dict(norm1=_norm(cfg, p + "norm1"), mixer=mixer, post1=_norm(cfg, p + "norm1b"))
        if layer.mlp is None:
            layers.append(LayerSpec(block="sandwich_mixer_only", position=position, **parts))
        else:
            layers.append(LayerSpec(block="sandwich", position=position, norm2=_norm(cfg, p + "norm2"),
                                    feed_forward=_feed_forward(cfg, layer.mlp, p + "mlp."), post2=_norm(cfg, p + "norm2b"),
                                    **parts))
    n = len(layers)
    order, steps = [], []
    if cfg.loop_times:
        order += [LayerCall(i) for i in range(cfg.loop_start)]
        for _ in range(cfg.loop_times):
            steps.append((len(order), PartSpec("pass_mix", dict(width=cfg.width, weight_name="loop.in"))))
            order += [LayerCall(i) for i in range(cfg.loop_start, cfg.loop_stop)]
        order += [LayerCall(i) for i in range(cfg.loop_stop, n)]
    else:
        order = [LayerCall(i) for i in range(n)]
    return ModelSpec(
        vocab_size=cfg.vocab, width=cfg.width,
        embedding=PartSpec("table", dict(vocab=cfg.vocab, width=cfg.width, weight_name="embed")),
        layers=tuple(layers), order=tuple(order), stream_steps=tuple(steps),
        final_norm=_norm(cfg, "final.norm"),
        head=PartSpec("linear", dict(vocab=cfg.vocab, width=cfg.width, weight_name=None)),
    )


def ignorable(cfg: SezanexConfig, name: str) -> bool:
    return False
