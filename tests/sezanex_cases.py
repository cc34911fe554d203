"""Small Sezanex configurations and model folders with random weights, for the tests."""

from __future__ import annotations

import json
import os

import torch
from safetensors.torch import save_file

from tt_transformers_b200.weights import random_tensors


def attention(heads, kv_heads, dim, vdim, window, rot_dims, base=1000.0, scaling=None, scale=None):
    m = {"heads": heads, "kv_heads": kv_heads, "dim": dim, "vdim": vdim, "scale": scale if scale is not None else dim ** -0.5}
    if window is not None:
        m["mask"] = {"size": window}
    if rot_dims:
        m["rot"] = {"base": base, "dims": rot_dims}
        if scaling is not None:
            factor, original, fast, slow = scaling
            m["rot"]["scaling"] = {"factor": factor, "original": original, "fast": fast, "slow": slow}
    return {"type": "attention", "mixer": m}


def mamba2(heads, vdim, state, groups, norm_groups, taps):
    return {"type": "mamba2", "mixer": {"heads": heads, "vdim": vdim, "state": state, "groups": groups,
                                        "norm_groups": norm_groups, "conv": taps}}


def dense(ff):
    return {"kind": "dense", "ff": ff}


def moe(experts, top, ff):
    return {"kind": "moe", "expert": {"ff": ff}, "router": {"experts": experts, "top": top}}


def layer(mixer, mlp):
    return dict(mixer, mlp=mlp)


def config(width, vocab, layers, loop, eps=1e-5):
    cfg = {"architecture": "Sezanex", "vocab": vocab, "width": width, "norm": {"eps": eps}, "layers": layers}
    if loop is not None:
        cfg["loop"] = {"start": loop[0], "stop": loop[1], "times": loop[2]}
    return cfg


# even sizes; a loop in the middle that runs three times; both mixers, every kind of feed-forward and none; a rotation
# over a part of the head with blended frequencies whose blend lies inside the head; key, value and state sizes that differ
ALIGNED = config(128, 300, [
    layer(attention(4, 2, 32, 16, window=24, rot_dims=16, scaling=(4.0, 64, 8.0, 1.0)), dense(160)),
    layer(mamba2(4, 16, 24, 2, 1, 4), moe(8, 2, 48)),
    layer(attention(6, 1, 16, 48, window=9, rot_dims=16, base=200.0, scaling=(2.0, 32, 4.0, 0.5)), None),
    layer(mamba2(2, 48, 8, 1, 4, 3), moe(6, 3, 32)),
], loop=(1, 3, 3))

# odd sizes and ones: one head, one group, one tap, one expert, a window of one position, no rotation scaling, a state of
# one number, all experts chosen, a loop that runs once and starts at the first layer
ODD = config(60, 131, [
    layer(mamba2(1, 6, 5, 1, 1, 1), moe(1, 1, 20)),
    layer(attention(1, 1, 10, 7, window=7, rot_dims=6, base=300.0), moe(9, 1, 9)),
    layer(attention(5, 5, 6, 9, window=1, rot_dims=2, scale=0.7), dense(33)),
    layer(mamba2(3, 5, 1, 3, 3, 6), moe(3, 3, 11)),
    layer(mamba2(6, 7, 3, 2, 2, 2), None),
], loop=(0, 2, 1), eps=1e-6)

# no loop at all (and no matrix at a pass's start), a window longer than any test prompt (plain causal attention with
# the constant in the denominator), no rotation in one layer, taps longer than most portions
PLAIN = config(64, 200, [
    layer(attention(2, 1, 24, 24, window=4096, rot_dims=24), moe(4, 2, 24)),
    layer(mamba2(2, 12, 16, 2, 2, 9), dense(96)),
    layer(attention(2, 2, 8, 8, window=None, rot_dims=0), None),
], loop=None)

# head sizes that the tensor-core kernels take (keys and values of 64), a window that ends inside a key tile, states
# of 64 x 64 and 128 x 32, a loop over all layers
TENSOR = config(128, 260, [
    layer(attention(4, 2, 64, 64, window=40, rot_dims=32, scaling=(8.0, 128, 16.0, 1.0)), moe(6, 2, 64)),
    layer(mamba2(2, 64, 64, 1, 2, 4), dense(192)),
    layer(mamba2(4, 32, 128, 2, 1, 4), None),
], loop=(0, 3, 2))


# keys and values of 128 (the other head size of the tensor-core attention), more query heads per key head, a window
# longer than a key tile, a wide state with few heads, the looped range at the end
WIDE = config(96, 180, [
    layer(mamba2(1, 128, 16, 1, 1, 3), moe(5, 3, 48)),
    layer(attention(4, 1, 128, 128, window=70, rot_dims=128, base=5000.0, scaling=(2.0, 64, 16.0, 2.0)), dense(96)),
    layer(mamba2(4, 16, 48, 4, 2, 4), None),
], loop=(1, 3, 2))


def single(kind):
    """One layer with one mechanism and nothing beside it."""
    if kind == "attention":
        layers = [layer(attention(4, 2, 12, 20, window=10, rot_dims=8, scaling=(3.0, 16, 4.0, 1.0)), None)]
    elif kind == "mamba2":
        layers = [layer(mamba2(4, 10, 6, 2, 2, 4), None)]
    elif kind == "dense":
        layers = [layer(mamba2(1, 8, 4, 1, 1, 2), dense(72))]
    elif kind == "moe":
        layers = [layer(mamba2(1, 8, 4, 1, 1, 2), moe(12, 3, 20))]
    else:
        raise KeyError(kind)
    return config(48, 97, layers, loop=None)


def write_folder(folder, cfg, seed, dtype=torch.float32):
    """Random weights: matrices N(0, 1/sqrt(columns)) so that every product keeps its scale; norm weights around one,
    their biases and slopes spread out so that leaving one out shows; decay rates from slow to fast, step-size biases and
    skips of both signs; routers with clear choices."""
    os.makedirs(folder, exist_ok=True)
    tensors = random_tensors(cfg, seed, std=1.0, norm_std=0.2, dtype=torch.float32)
    gen = torch.Generator().manual_seed(seed + 1)
    for name, t in tensors.items():
        if name.endswith(".alpha"):
            tensors[name] = torch.rand((), generator=gen) * 0.8 + 0.3
        elif name.endswith(".b"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.3
        elif name.endswith(".A_log"):
            tensors[name] = torch.rand(t.shape, generator=gen) * 4.0 - 3.0        # rates from 0.05 to 2.7
        elif name.endswith(".dt_bias"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 1.5 - 0.5
        elif name.endswith(".D"):
            tensors[name] = torch.randn(t.shape, generator=gen)
        elif name.endswith(".conv"):
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.5
        elif t.dim() >= 2:
            tensors[name] = t * t.shape[-1] ** -0.5
        if name.endswith(".router"):
            tensors[name] = tensors[name] * 4.0           # scores spread out, so that the chosen experts are seldom nearly tied
        if name == "loop.in":
            tensors[name] = tensors[name] * 1.4           # two inputs of unit scale: keep the stream's scale
    tensors = {k: v.to(dtype).contiguous() for k, v in tensors.items()}
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    save_file(tensors, os.path.join(folder, "model.safetensors"))
    return folder


def read_folder(folder):
    from safetensors import safe_open

    with open(os.path.join(folder, "config.json")) as f:
        cfg = json.load(f)
    w = {}
    with safe_open(os.path.join(folder, "model.safetensors"), framework="pt", device="cpu") as f:
        for name in f.keys():
            w[name] = f.get_tensor(name).to(torch.float32)
    return cfg, w
