"""What the command lines share: named random models and loading."""

from __future__ import annotations

import tempfile

import torch

LLAMA3_SCALING = {"rope_type": "llama3", "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                  "original_max_position_embeddings": 8192}


def llama_config(hidden, layers, heads, kv_heads, head_dim, inter, factor, tied, vocab=128256):
    return {"architectures": ["LlamaForCausalLM"], "hidden_size": hidden, "num_hidden_layers": layers,
            "num_attention_heads": heads, "num_key_value_heads": kv_heads, "head_dim": head_dim,
            "intermediate_size": inter, "vocab_size": vocab, "rms_norm_eps": 1e-5, "max_position_embeddings": 131072,
            "rope_theta": 500000.0, "rope_scaling": dict(LLAMA3_SCALING, factor=factor), "tie_word_embeddings": tied}


# Layer sizes of the models that the reference ships packages for (src/tt_transformers/models/
# llama32_1b, llama32_3b, llama3_8b), for runs with random weights where no checkpoint is at hand.
RANDOM_MODELS = {
    "llama-3.2-1b": llama_config(2048, 16, 32, 8, 64, 8192, 32.0, True),
    "llama-3.2-3b": llama_config(3072, 28, 24, 8, 128, 8192, 32.0, True),
    "llama-3.1-8b": llama_config(4096, 32, 32, 8, 128, 14336, 8.0, False),
    "tiny": {"architectures": ["LlamaForCausalLM"], "hidden_size": 128, "num_hidden_layers": 2,
             "num_attention_heads": 8, "num_key_value_heads": 2, "head_dim": 64, "intermediate_size": 256,
             "vocab_size": 512, "rms_norm_eps": 1e-5, "max_position_embeddings": 4096, "rope_theta": 10000.0,
             "tie_word_embeddings": True},
}


def bozavik_config(width, layers, heads, dim, rot_dim, vdim, q_rank, kv_rank, experts, top, ff, shared_ff, vocab):
    """Layers alternate between the two latent-attention mixers; every layer has the routed feed-forward."""
    def mixer(second):
        m = {"heads": heads, "dim": dim, "vdim": vdim, "q_rank": q_rank, "kv_rank": kv_rank,
             "scale": (dim + (rot_dim if second else 0)) ** -0.5}
        if second:
            m.update(rot_dim=rot_dim, rot={"base": 10000.0, "dims": rot_dim})
        return m

    mlp = {"kind": "moe", "router": {"experts": experts, "top": top}, "expert": {"ff": ff, "limit": 7.0},
           "shared": {"ff": shared_ff, "limit": 7.0}}
    return {"architecture": "Bozavik", "vocab": vocab, "width": width, "residual_mult": 0.7, "norm": {"eps": 1e-5},
            "embedding": {"scale": 1.0},
            "layers": [{"type": "latent_attention_2" if i % 2 else "latent_attention", "mixer": mixer(i % 2 == 1),
                        "mlp": mlp} for i in range(layers)]}


def pedazen_config(width, pairs, lightning_heads, heads, kv_heads, head_dim, chunk, channels, blocks, experts, top, ff, groups,
                   keep, dense_ff, vocab, loop=None):
    """`pairs` times a linear-attention layer followed by a layer with softmax attention and a recurrent block side
    by side; the first layer has a dense feed-forward, the others routed experts."""
    def lightning():
        decay = [1.0 - 2.0 ** (-3 - 5 * h / max(1, lightning_heads - 1)) for h in range(lightning_heads)]
        return {"type": "lightning", "mixer": {"heads": lightning_heads, "dim": head_dim, "vdim": head_dim, "decay": decay}}

    def parallel():
        left = {"heads": heads, "kv_heads": kv_heads, "dim": head_dim, "vdim": head_dim, "mask": {"size": chunk},
                "rot": {"base": 10000.0, "dims": head_dim // 2}, "scale": head_dim ** -0.5, "softcap": 30.0}
        return {"type": "parallel", "mixer": {"left": left, "right": {"width": channels, "blocks": blocks, "conv": 4}}}

    moe = {"kind": "moe", "expert": {"ff": ff}, "router": {"experts": experts, "top": top, "groups": {"count": groups, "keep": keep}}}
    layers = []
    for i in range(pairs):
        layers.append(dict(lightning(), mlp={"kind": "dense", "ff": dense_ff} if i == 0 else moe))
        layers.append(dict(parallel(), mlp=moe))
    cfg = {"architecture": "Pedazen", "vocab": vocab, "width": width, "norm": {"eps": 1e-6}, "embedding": {"scale": 1.0},
           "layers": layers}
    if loop:
        cfg["loop"] = {"start": loop[0], "stop": loop[1], "times": loop[2]}
    return cfg


def sezanex_config(width, blocks, ssm_heads, ssm_vdim, state, ssm_groups, heads, kv_heads, head_dim, window, experts, top, ff,
                   dense_ff, vocab, loop=None):
    """`blocks` times three state-space layers followed by one layer of windowed softmax attention; the first layer
    has a dense feed-forward, the others scored experts."""
    def mamba2():
        return {"type": "mamba2", "mixer": {"heads": ssm_heads, "vdim": ssm_vdim, "state": state, "groups": ssm_groups,
                                            "norm_groups": ssm_groups, "conv": 4}}

    def attention():
        return {"type": "attention", "mixer": {
            "heads": heads, "kv_heads": kv_heads, "dim": head_dim, "vdim": head_dim, "mask": {"size": window},
            "rot": {"base": 10000.0, "dims": head_dim, "scaling": {"factor": 4.0, "original": 4096, "fast": 32.0, "slow": 1.0}},
            "scale": head_dim ** -0.5}}

    moe = {"kind": "moe", "expert": {"ff": ff}, "router": {"experts": experts, "top": top}}
    layers = []
    for i in range(blocks):
        for j in range(3):
            layers.append(dict(mamba2(), mlp={"kind": "dense", "ff": dense_ff} if i == 0 and j == 0 else moe))
        layers.append(dict(attention(), mlp=moe))
    cfg = {"architecture": "Sezanex", "vocab": vocab, "width": width, "norm": {"eps": 1e-5}, "layers": layers}
    if loop:
        cfg["loop"] = {"start": loop[0], "stop": loop[1], "times": loop[2]}
    return cfg


def bufolorn_config(width, blocks, heads, kv_heads, head_dim, state_heads, state_dim, latent_heads, latent_dim, rot_dim, latent_vdim,
                    kv_rank, window, delta_heads, delta_kv_heads, delta_dim, delta_vdim, experts, top, ff, shared_ff, dense_ff, vocab):
    """`blocks` times four layers: softmax attention with a distance bias beside a token-shift state (dense feed-forward),
    latent attention over a window, a delta rule with channel decays, and latent attention that reads the latent of the
    layer two before it (corrected experts with a shared one in all three)."""
    def side_by_side():
        left = {"heads": heads, "kv_heads": kv_heads, "dim": head_dim, "vdim": head_dim, "scale": head_dim ** -0.5 * 4, "softcap": 30.0,
                "bias_max": 1024, "bias_rows": 32, "q_temp": {"coef": 0.3, "every": 1024}}
        return {"type": "parallel", "mixer": {"left": left, "right": {"heads": state_heads, "dim": state_dim, "decay_rank": 64},
                                              "left_scale": 0.5, "right_scale": 0.5}}

    def latent(kv_from=None):
        m = {"heads": latent_heads, "dim": latent_dim, "rot_dim": rot_dim, "vdim": latent_vdim, "kv_rank": kv_rank,
             "scale": (latent_dim + rot_dim) ** -0.5, "mask": {"size": window},
             "rot": {"base": 10000.0, "dims": rot_dim, "scaling": {"factor": 4.0, "original": 4096, "fast": 32.0, "slow": 1.0}}}
        if kv_from is not None:
            m["kv_from"] = kv_from
        return {"type": "latent_attention", "mixer": m}

    def delta():
        return {"type": "channel_delta", "mixer": {"heads": delta_heads, "kv_heads": delta_kv_heads, "dim": delta_dim, "vdim": delta_vdim,
                                                   "conv": 4, "decay_rank": 64, "gate_rank": 64}}

    moe = {"kind": "moe", "expert": {"ff": ff}, "router": {"experts": experts, "top": top, "scale": 1.0}, "shared": {"ff": shared_ff}}
    layers = []
    for b in range(blocks):
        layers += [dict(side_by_side(), mlp={"kind": "dense", "ff": dense_ff}), dict(latent(), mlp=moe), dict(delta(), mlp=moe),
                   dict(latent(kv_from=4 * b + 1), mlp=moe)]
    return {"architecture": "Bufolorn", "vocab": vocab, "width": width, "residual_mult": 0.5, "norm": {"eps": 1e-5},
            "embedding": {"scale": 1.0}, "layers": layers}


def layer_runs(cfg: dict) -> int:
    """How many layers a token passes in a configuration with a `loop`, looped layers counted every time."""
    loop = cfg.get("loop")
    return len(cfg["layers"]) + ((loop["stop"] - loop["start"]) * (loop["times"] - 1) if loop else 0)


def closest_llama(cfg: dict) -> dict:
    """The dense decoder of this package that is closest to a configuration of another design: the same width,
    depth and vocabulary. For Bozavik: the same heads (head size = unrotated + rotated query elements), one KV
    head per four heads, and a feed-forward as wide as the experts a token uses plus the shared one. For Pedazen:
    as many layers as a token passes, the heads, KV heads and head size of its softmax attention, and a
    feed-forward as wide as the experts a token uses. For Sezanex: the same with its windowed attention's heads. For
    Bufolorn: the heads of its softmax attention, and a feed-forward as wide as the experts a token uses plus the shared one."""
    if cfg.get("architecture") == "Bufolorn":
        a = next(l["mixer"]["left"] for l in cfg["layers"] if l["type"] == "parallel")
        f = next(l["mlp"] for l in cfg["layers"] if l["mlp"] and l["mlp"]["kind"] == "moe")
        inter = f["router"]["top"] * f["expert"]["ff"] + (f.get("shared") or {}).get("ff", 0)
        return {"architectures": ["LlamaForCausalLM"], "hidden_size": cfg["width"], "num_hidden_layers": len(cfg["layers"]),
                "num_attention_heads": a["heads"], "num_key_value_heads": a["kv_heads"], "head_dim": a["dim"],
                "intermediate_size": inter, "vocab_size": cfg["vocab"], "rms_norm_eps": 1e-5,
                "max_position_embeddings": 131072, "rope_theta": 500000.0, "tie_word_embeddings": False}
    if cfg.get("architecture") == "Sezanex":
        a = next(l["mixer"] for l in cfg["layers"] if l["type"] == "attention")
        f = next(l["mlp"] for l in cfg["layers"] if l["mlp"] and l["mlp"]["kind"] == "moe")
        return {"architectures": ["LlamaForCausalLM"], "hidden_size": cfg["width"], "num_hidden_layers": layer_runs(cfg),
                "num_attention_heads": a["heads"], "num_key_value_heads": a["kv_heads"], "head_dim": a["dim"],
                "intermediate_size": f["router"]["top"] * f["expert"]["ff"], "vocab_size": cfg["vocab"], "rms_norm_eps": 1e-5,
                "max_position_embeddings": 131072, "rope_theta": 500000.0, "tie_word_embeddings": True}
    if cfg.get("architecture") == "Pedazen":
        left = next(l["mixer"]["left"] for l in cfg["layers"] if l["type"] == "parallel")
        f = next(l["mlp"] for l in cfg["layers"] if l["mlp"] and l["mlp"]["kind"] == "moe")
        return {"architectures": ["LlamaForCausalLM"], "hidden_size": cfg["width"], "num_hidden_layers": layer_runs(cfg),
                "num_attention_heads": left["heads"], "num_key_value_heads": left["kv_heads"], "head_dim": left["dim"],
                "intermediate_size": f["router"]["top"] * f["expert"]["ff"], "vocab_size": cfg["vocab"], "rms_norm_eps": 1e-5,
                "max_position_embeddings": 131072, "rope_theta": 500000.0, "tie_word_embeddings": True}
    layer = cfg["layers"][-1]
    m, f = layer["mixer"], layer["mlp"]
    heads, head_dim = m["heads"], m["dim"] + m.get("rot_dim", 0)
    inter = f["router"]["top"] * f["expert"]["ff"] + (f.get("shared") or {}).get("ff", 0)
    return {"architectures": ["LlamaForCausalLM"], "hidden_size": cfg["width"], "num_hidden_layers": len(cfg["layers"]),
            "num_attention_heads": heads, "num_key_value_heads": max(1, heads // 4), "head_dim": head_dim,
            "intermediate_size": inter, "vocab_size": cfg["vocab"], "rms_norm_eps": 1e-5,
            "max_position_embeddings": 131072, "rope_theta": 500000.0, "tie_word_embeddings": False}


RANDOM_MODELS.update({
    "bozavik-tiny": bozavik_config(128, 2, 4, 16, 16, 16, 64, 64, 4, 2, 64, 64, 512),
    "bozavik-a": bozavik_config(1024, 8, 16, 32, 32, 64, 384, 128, 16, 4, 512, 1024, 32768),
    "bozavik-b": bozavik_config(2048, 8, 16, 64, 64, 128, 768, 256, 32, 4, 1024, 2048, 65536),
})


RANDOM_MODELS.update({
    "pedazen-tiny": pedazen_config(128, 1, 2, 4, 2, 64, 64, 128, 2, 4, 2, 64, 2, 1, 256, 512, loop=(0, 2, 2)),
    "pedazen-a": pedazen_config(1024, 4, 8, 16, 4, 64, 1024, 1024, 8, 16, 4, 512, 4, 2, 2048, 32768, loop=(2, 4, 2)),
    "pedazen-b": pedazen_config(2048, 4, 16, 16, 4, 128, 2048, 2048, 8, 32, 4, 1024, 8, 4, 4096, 65536, loop=(2, 4, 2)),
})


RANDOM_MODELS.update({
    "sezanex-tiny": sezanex_config(128, 1, 4, 32, 32, 2, 4, 2, 64, 64, 4, 2, 64, 256, 512, loop=(1, 4, 2)),
    "sezanex-a": sezanex_config(1024, 2, 32, 64, 128, 2, 16, 4, 64, 1024, 16, 4, 512, 2048, 32768, loop=(2, 4, 2)),
    "sezanex-b": sezanex_config(2048, 2, 64, 64, 128, 4, 16, 4, 128, 2048, 32, 4, 1024, 4096, 65536, loop=(2, 4, 2)),
})


RANDOM_MODELS.update({
    "bufolorn-tiny": bufolorn_config(128, 1, 4, 2, 64, 2, 32, 4, 16, 16, 32, 64, 64, 4, 2, 32, 32, 4, 2, 64, 64, 256, 512),
    "bufolorn-a": bufolorn_config(1024, 2, 16, 4, 64, 16, 64, 16, 32, 32, 64, 128, 1024, 16, 4, 64, 64, 16, 4, 512, 512, 2048, 32768),
    "bufolorn-b": bufolorn_config(2048, 2, 16, 4, 128, 32, 64, 16, 64, 64, 128, 256, 2048, 16, 4, 128, 128, 32, 4, 1024, 1024, 4096, 65536),
})


def load(hf_model, random_model, *, seed=0, **engine_options):
    """An LLM from a model folder, or from a named random model (weights drawn on the GPU)."""
    from ..config.engine import EngineConfig
    from ..engine.llm import LLM, from_pretrained
    from ..engine.step import build_engine
    from ..weights import random_tensors

    if hf_model:
        return from_pretrained(hf_model, **engine_options)
    if random_model not in RANDOM_MODELS:
        raise SystemExit(f"unknown random model {random_model!r}; known: {sorted(RANDOM_MODELS)}")
    cfg = RANDOM_MODELS[random_model]
    n_layers = engine_options.pop("n_layers", None)
    device = engine_options.get("device", "cuda:0")
    tensors = random_tensors(cfg, seed=seed, dtype=torch.bfloat16, device=device)
    engine = build_engine(config_dict=cfg, tensors=tensors, engine_config=EngineConfig(**engine_options),
                          n_layers=n_layers)
    return LLM(engine)
