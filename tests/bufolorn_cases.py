"""Small Bufolorn configurations and model folders with random weights, for the tests."""

from __future__ import annotations

import copy
import json
import os

import torch
from safetensors.torch import save_file

from tt_transformers_b200.weights import random_tensors


def delta(heads, kv_heads, dim, vdim, taps, decay_rank=5, gate_rank=7):
    return {"type": "channel_delta", "mixer": {"heads": heads, "kv_heads": kv_heads, "dim": dim, "vdim": vdim, "conv": taps,
                                               "decay_rank": decay_rank, "gate_rank": gate_rank}}


def side_by_side(heads, kv_heads, dim, vdim, bias_rows, bias_max, state_heads, state_dim, scale=None, softcap=15.0, temp=(0.4, 8),
                 left_scale=0.7, right_scale=0.4, decay_rank=6):
    left = {"heads": heads, "kv_heads": kv_heads, "dim": dim, "vdim": vdim, "scale": scale if scale is not None else dim ** -0.5 * 2,
            "bias_max": bias_max, "bias_rows": bias_rows}
    if softcap is not None:
        left["softcap"] = softcap
    if temp is not None:
        left["q_temp"] = {"coef": temp[0], "every": temp[1]}
    return {"type": "parallel", "mixer": {"left": left, "right": {"heads": state_heads, "dim": state_dim, "decay_rank": decay_rank},
                                          "left_scale": left_scale, "right_scale": right_scale}}


def latent(heads, dim, rot_dim, vdim, kv_rank, window, base=500.0, scaling=None, scale=None, kv_from=None, rot_dims=None):
    m = {"heads": heads, "dim": dim, "rot_dim": rot_dim, "vdim": vdim, "kv_rank": kv_rank,
         "scale": scale if scale is not None else (dim + rot_dim) ** -0.5}
    if window is not None:
        m["mask"] = {"size": window}
    if rot_dim:
        m["rot"] = {"base": base, "dims": rot_dims if rot_dims is not None else rot_dim}
        if scaling is not None:
            factor, original, fast, slow = scaling
            m["rot"]["scaling"] = {"factor": factor, "original": original, "fast": fast, "slow": slow}
    if kv_from is not None:
        m["kv_from"] = kv_from
    return {"type": "latent_attention", "mixer": m}


def dense(ff):
    return {"kind": "dense", "ff": ff}


def moe(experts, top, ff, scale=1.0, shared=None):
    f = {"kind": "moe", "expert": {"ff": ff}, "router": {"experts": experts, "top": top, "scale": scale}}
    if shared is not None:
        f["shared"] = {"ff": shared}
    return f


def layer(mixer, mlp):
    return dict(mixer, mlp=mlp)


def config(width, vocab, layers, eps=1e-5, mult=0.5, embed=3.0):
    cfg = {"architecture": "Bufolorn", "vocab": vocab, "width": width, "norm": {"eps": eps}, "layers": layers,
           "residual_mult": mult}
    if embed is not None:
        cfg["embedding"] = {"scale": embed}
    return cfg


# even sizes; every mixer and every feed-forward, and a layer without one; a layer that reads another layer's latent through
# a wider window than the owner's; a distance table whose logarithmic rows are reached inside the test prompts; a query
# temperature that changes every eight positions
ALIGNED = config(128, 300, [
    layer(side_by_side(4, 2, 32, 16, bias_rows=12, bias_max=40, state_heads=2, state_dim=24), dense(160)),
    layer(latent(4, 16, 16, 24, 48, window=24, scaling=(4.0, 64, 8.0, 1.0)), moe(8, 2, 48, scale=1.3, shared=64)),
    layer(delta(4, 2, 16, 24, taps=4), moe(6, 3, 32, scale=0.8)),
    layer(latent(2, 24, 16, 8, 48, window=40, scaling=(4.0, 64, 8.0, 1.0), kv_from=1), None),
    layer(side_by_side(6, 1, 16, 48, bias_rows=8, bias_max=300, state_heads=4, state_dim=8, softcap=None, temp=None), dense(96)),
])

# odd sizes and ones: one head, one tap, one expert, a window of one position, a distance table with an odd number of rows
# and one with two, a rotation over a part of the rotated part, no rotation scaling, no rotated part at all, all experts
# chosen, multipliers of one, a decay of rank one
ODD = config(60, 131, [
    layer(delta(1, 1, 6, 10, taps=1, decay_rank=1, gate_rank=1), moe(1, 1, 20)),
    layer(latent(1, 10, 6, 7, 9, window=7, base=300.0, rot_dims=4), moe(9, 1, 9, shared=5)),
    layer(side_by_side(5, 5, 6, 9, bias_rows=5, bias_max=9, state_heads=1, state_dim=5, scale=0.7, temp=(1.0, 1), left_scale=1.0,
                       right_scale=1.0, decay_rank=1), dense(33)),
    layer(latent(5, 6, 0, 9, 11, window=1), moe(3, 3, 11, scale=2.0)),
    layer(delta(6, 2, 3, 7, taps=2), None),
    layer(latent(3, 4, 6, 5, 9, window=None, base=300.0, rot_dims=4, kv_from=1), dense(21)),
    layer(side_by_side(2, 1, 10, 4, bias_rows=2, bias_max=3, state_heads=3, state_dim=7), None),
], eps=1e-6, mult=1.0, embed=None)

# head sizes that the tensor-core kernels take (keys and values of 64 and 128, a latent of 64 with a rotated part of 32),
# windows that end inside a key tile, states of 64 x 64 and 128 x 32
TENSOR = config(128, 260, [
    layer(side_by_side(4, 2, 64, 64, bias_rows=16, bias_max=100, state_heads=2, state_dim=64), moe(6, 2, 64, shared=32)),
    layer(latent(4, 32, 32, 16, 64, window=40, scaling=(8.0, 128, 16.0, 1.0)), dense(192)),
    layer(delta(2, 1, 64, 64, taps=3), None),
    layer(delta(4, 4, 128, 32, taps=4), dense(64)),
    layer(latent(8, 16, 32, 32, 64, window=33, scaling=(8.0, 128, 16.0, 1.0), kv_from=1), None),
    layer(side_by_side(2, 1, 128, 128, bias_rows=6, bias_max=20, state_heads=1, state_dim=32, temp=(0.3, 100)), None),
], mult=0.7)


def single(kind):
    """One layer with one mechanism and as little as can be beside it."""
    tiny = delta(1, 1, 4, 4, taps=1, decay_rank=2, gate_rank=2)
    if kind == "delta":
        layers = [layer(delta(4, 2, 6, 10, taps=3), None)]
    elif kind == "side_by_side":
        layers = [layer(side_by_side(4, 2, 12, 20, bias_rows=10, bias_max=25, state_heads=3, state_dim=6), None)]
    elif kind == "latent":
        layers = [layer(latent(4, 12, 8, 20, 24, window=10, scaling=(3.0, 16, 4.0, 1.0)), None)]
    elif kind == "shared_latent":
        layers = [layer(latent(2, 6, 8, 10, 24, window=6, scaling=(3.0, 16, 4.0, 1.0)), None),
                  layer(latent(3, 10, 8, 4, 24, window=13, scaling=(3.0, 16, 4.0, 1.0), kv_from=0), None)]
    elif kind == "dense":
        layers = [layer(tiny, dense(72))]
    elif kind == "moe":
        layers = [layer(tiny, moe(12, 3, 20, scale=1.7, shared=16))]
    else:
        raise KeyError(kind)
    return config(48, 97, layers)


def without_sizes_of_made_up_tensors(cfg):
    """The configuration as a checkpoint's author writes it: ranks and table rows are in the tensors' shapes only."""
    cfg = copy.deepcopy(cfg)
    for entry in cfg["layers"]:
        for m in (entry["mixer"], entry["mixer"].get("left", {}), entry["mixer"].get("right", {})):
            for key in ("decay_rank", "gate_rank", "bias_rows"):
                m.pop(key, None)
    return cfg


def write_folder(folder, cfg, seed, dtype=torch.float32, keep_sizes=False):
    """Random weights: matrices N(0, 1/sqrt(columns)) so that every product keeps its scale; norm weights around one, biases
    spread out so that leaving one out shows; decay rates from slow to fast, step-size biases of both signs, mixing weights
    between 0 and 1, sinks and distance rows of a size that matters beside the scores, corrections that change choices."""
    os.makedirs(folder, exist_ok=True)
    tensors = random_tensors(cfg, seed, std=1.0, norm_std=0.2, dtype=torch.float32)
    gen = torch.Generator().manual_seed(seed + 1)
    for name, t in tensors.items():
        last = name.rsplit(".", 1)[-1]
        if last == "b" and t.dim() == 1:
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.3
        elif last == "A_log":
            tensors[name] = torch.rand(t.shape, generator=gen) * 4.0 - 3.0        # rates from 0.05 to 2.7
        elif last == "dt_bias":
            tensors[name] = torch.randn(t.shape, generator=gen) * 1.5 - 0.5
        elif last == "w0":
            tensors[name] = torch.randn(t.shape, generator=gen) * 1.5 - 1.5       # decays from nearly one to nearly none
        elif last == "conv":
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.5
        elif last == "u" and ".right." in name:
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.7
        elif ".mu." in name:
            tensors[name] = torch.rand(t.shape, generator=gen)
        elif last == "sink":
            tensors[name] = torch.randn(t.shape, generator=gen) * 2.0
        elif last == "rel":
            tensors[name] = torch.randn(t.shape, generator=gen) * 1.5
        elif last == "correction":
            tensors[name] = torch.randn(t.shape, generator=gen) * 0.3
        elif t.dim() >= 2:
            tensors[name] = t * t.shape[-1] ** -0.5
        if last == "router":
            tensors[name] = tensors[name] * 4.0           # scores spread out, so that the chosen experts are seldom nearly tied
    tensors = {k: v.to(dtype).contiguous() for k, v in tensors.items()}
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(cfg if keep_sizes else without_sizes_of_made_up_tensors(cfg), f, indent=1)
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


def random_config(seed):
    """A configuration drawn from a seed: sizes, head counts, layer order, windows, ranks, taps and constants all vary;
    layers that read another layer's latent appear where an owner with the same latent sizes stands before them."""
    import random

    rng = random.Random(seed)
    pick = rng.choice
    width = pick([40, 64, 96, 136, 200, 256])

    def some_mlp():
        kind = pick(["none", "dense", "moe", "moe"])
        if kind == "none":
            return None
        if kind == "dense":
            return dense(pick([24, 70, 128, 264]))
        experts = pick([1, 2, 5, 8, 12, 16])
        return moe(experts, rng.randint(1, min(experts, 4)), pick([8, 24, 40, 64]), scale=pick([1.0, 0.6, 2.5]),
                   shared=pick([None, 16, 56]))

    families = []                       # latent sizes that owners of a latent have used so far: (layer, kv_rank, rot_dim, rot keys)
    layers = []
    for i in range(rng.randint(2, 7)):
        kind = pick(["delta", "side", "latent", "latent"])
        if kind == "delta":
            kv = pick([1, 2, 3])
            mixer = delta(kv * pick([1, 2, 4]), kv, pick([4, 8, 24, 32, 64]), pick([8, 16, 40, 64]), taps=rng.randint(1, 5),
                          decay_rank=rng.randint(1, 24), gate_rank=rng.randint(1, 24))
        elif kind == "side":
            kv = pick([1, 2, 3])
            dim = pick([8, 16, 24, 64, 128])
            rows = pick([2, 4, 6, 10, 16, 32])
            mixer = side_by_side(kv * pick([1, 2, 4]), kv, dim, pick([dim, dim, 8, 48]), bias_rows=rows,
                                 bias_max=rows // 2 + rng.randint(1, 150), state_heads=rng.randint(1, 4), state_dim=pick([4, 8, 20, 32, 64]),
                                 scale=pick([None, 0.3, 1.1]), softcap=pick([None, 8.0, 30.0]), temp=pick([None, (0.5, 16), (0.2, 3)]),
                                 left_scale=pick([1.0, 0.6]), right_scale=pick([1.0, 0.45]), decay_rank=rng.randint(1, 20))
        else:
            heads, dim, vdim = pick([1, 2, 4, 5, 8]), pick([8, 16, 32, 64]), pick([8, 16, 24, 64])
            window = pick([None, 1, 5, 33, 64, 150])
            if families and rng.random() < 0.5:
                owner, kv_rank, rot_dim, rot = pick(families)
                mixer = latent(heads, dim, rot_dim, vdim, kv_rank, window, kv_from=owner)
                if rot is not None:
                    mixer["mixer"]["rot"] = copy.deepcopy(rot)
            else:
                rot_dim = pick([0, 4, 16, 32, 64])
                mixer = latent(heads, dim, rot_dim, vdim, pick([16, 24, 48, 64, 128]), window, base=pick([100.0, 10000.0]),
                               scaling=pick([None, (4.0, 64, 8.0, 1.0), (2.0, 32, 4.0, 0.5)]))
                families.append((i, mixer["mixer"]["kv_rank"], rot_dim, mixer["mixer"].get("rot")))
        layers.append(layer(mixer, some_mlp()))
    return config(width, rng.randint(50, 700), layers, eps=pick([1e-5, 1e-6]), mult=pick([1.0, 0.5, 0.8]), embed=pick([None, 2.0, 9.0]))
