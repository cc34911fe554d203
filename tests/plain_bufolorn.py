"""A plain, slow implementation of the Bufolorn decoder: one function per mechanism, whole sequences at once,
float64 unless told otherwise. It shares no code with the package; the tests compare the engine with it.

A model is (config dictionary, {tensor name: tensor}). Weights are [out, in] and applied as W x.

    embedding:   x = s_e E[token]
    layer:       h = LN(x);  x = x + m (mixer(h) + ff(h))            (one layer norm with a bias, both sub-layers read it)
    mixers:      `channel_delta` (a delta rule with a decay per key channel), `parallel` (softmax attention with a learned
                 distance bias beside a decayed outer-product state with token shift), `latent_attention` (keys and values
                 from a cached latent, a sliding window, optionally another layer's latent)
    output:      logits = W_head LN_final(x)
"""

import math

import torch

F = torch.float64


def layer_norm(x, weight, bias, eps):
    dev = x - x.mean(-1, keepdim=True)
    return dev / torch.sqrt((dev * dev).mean(-1, keepdim=True) + eps) * weight + bias


def rms(x, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)


def silu(z):
    return z * torch.sigmoid(z)


def softplus(z):
    return torch.where(z > 30, z, torch.log1p(torch.exp(torch.clamp(z, max=30))))


# ---------------------------------------------------------------------------- the delta rule with channel decays
def short_conv_silu(x, weight):
    """x [T, C]; weight [C, taps], the last column is the current token's; zeros before the start; no bias."""
    T, C = x.shape
    taps = weight.shape[1]
    padded = torch.cat([torch.zeros(taps - 1, C, dtype=x.dtype), x], 0)
    out = torch.zeros(T, C, dtype=x.dtype)
    for j in range(taps):
        out = out + padded[j:j + T] * weight[:, j]
    return silu(out)


def unit(x):
    return x / torch.sqrt((x * x).sum(-1, keepdim=True) + 1e-6)


def channel_delta(h, w, p, m, eps):
    T = h.shape[0]
    H, G, D, V = m["heads"], m["kv_heads"], m["dim"], m["vdim"]
    q = short_conv_silu(h @ w[p + "q"].T, w[p + "q.conv"]).view(T, G, D)
    k = short_conv_silu(h @ w[p + "k"].T, w[p + "k.conv"]).view(T, G, D)
    v = short_conv_silu(h @ w[p + "v"].T, w[p + "v.conv"]).view(T, H, V)
    q, k = unit(q) * D ** -0.5, unit(k)
    beta = torch.sigmoid(h @ w[p + "b"].T)                                                  # [T, H]
    step = softplus((h @ w[p + "a1"].T) @ w[p + "a2"].T + w[p + "dt_bias"]).view(T, H, D)
    decay = torch.exp(-torch.exp(w[p + "A_log"])[None, :, None] * step)                    # [T, H, D]
    out = torch.zeros(T, H, V, dtype=h.dtype)
    for head in range(H):
        g = head // (H // G)
        S = torch.zeros(D, V, dtype=h.dtype)
        for t in range(T):
            S = decay[t, head][:, None] * S
            u = beta[t, head] * (v[t, head] - S.T @ k[t, g])
            S = S + torch.outer(k[t, g], u)
            out[t, head] = S.T @ q[t, g]
    gate = torch.sigmoid((h @ w[p + "g1"].T) @ w[p + "g2"].T).view(T, H, V)
    out = rms(out, eps) * w[p + "norm"] * gate
    return out.reshape(T, H * V) @ w[p + "o"].T


# ---------------------------------------------------------------------------- attention with a distance bias
def distance_bucket(n, rows, far):
    half = rows // 2
    if n < half:
        return n
    return min(rows - 1, half + int(math.floor(math.log(n / half) / math.log(far / half) * (rows - half))))


def biased_attention(h, w, p, m, eps):
    T = h.shape[0]
    H, G, D, V = m["heads"], m["kv_heads"], m["dim"], m["vdim"]
    q = rms((h @ w[p + "q"].T + w[p + "q.b"]).view(T, H, D), eps)
    k = rms((h @ w[p + "k"].T + w[p + "k.b"]).view(T, G, D), eps)
    v = (h @ w[p + "v"].T + w[p + "v.b"]).view(T, G, V)
    t = m.get("q_temp")
    if t:
        pos = torch.arange(T)
        q = q * (1 + t["coef"] * torch.log(torch.floor((pos + 1) / t["every"]).to(h.dtype) + 1))[:, None, None]
    rel = w[p + "rel"]
    rows = rel.shape[0]
    cap = m.get("softcap")
    out = torch.zeros(T, H, V, dtype=h.dtype)
    for head in range(H):
        g = head // (H // G)
        for i in range(T):
            s = (k[:i + 1, g] @ q[i, head]) * m["scale"]
            if cap:
                s = cap * torch.tanh(s / cap)
            s = s + torch.stack([rel[distance_bucket(i - j, rows, m["bias_max"]), head] for j in range(i + 1)])
            top = torch.maximum(s.max(), w[p + "sink"][head])
            e = torch.exp(s - top)
            out[i, head] = (e / (e.sum() + torch.exp(w[p + "sink"][head] - top))) @ v[:i + 1, g]
    return out.reshape(T, H * V) @ w[p + "o"].T + w[p + "o.b"]


# ---------------------------------------------------------------------------- the decayed outer-product state
def shifted_state(h, w, p, m, eps):
    T = h.shape[0]
    H, D = m["heads"], m["dim"]
    before = torch.cat([torch.zeros(1, h.shape[1], dtype=h.dtype), h[:-1]], 0)

    def mix(name):
        return h + (before - h) * w[p + "mu." + name]

    r = (mix("r") @ w[p + "r"].T).view(T, H, D)
    k = (mix("k") @ w[p + "k"].T).view(T, H, D)
    v = (mix("v") @ w[p + "v"].T).view(T, H, D)
    gate = silu(mix("g") @ w[p + "g"].T)
    decay = torch.exp(-torch.exp(torch.tanh(mix("w") @ w[p + "w1"].T) @ w[p + "w2"].T + w[p + "w0"])).view(T, H, D)
    out = torch.zeros(T, H, D, dtype=h.dtype)
    for head in range(H):
        S = torch.zeros(D, D, dtype=h.dtype)
        for t in range(T):
            kv = torch.outer(k[t, head], v[t, head])
            out[t, head] = (S + w[p + "u"][head][:, None] * kv).T @ r[t, head]
            S = decay[t, head][:, None] * S + kv
    out = rms(out, eps).reshape(T, H * D) * w[p + "norm"] * gate
    return out @ w[p + "o"].T


def side_by_side(h, w, p, m, eps):
    return (m["left_scale"] * biased_attention(h, w, p + "left.", m["left"], eps)
            + m["right_scale"] * shifted_state(h, w, p + "right.", m["right"], eps))


# ---------------------------------------------------------------------------- attention over a latent
def blended_frequencies(rot, dtype=F):
    dims, base = rot["dims"], rot["base"]
    f = [base ** (-2.0 * i / dims) for i in range(dims // 2)]
    sc = rot.get("scaling")
    if not sc:
        return torch.tensor(f, dtype=dtype), 1.0

    def turn(t):
        return dims * math.log(sc["original"] / (2 * math.pi * t)) / (2 * math.log(base))

    lo = max(math.floor(turn(sc["fast"])), 0)
    hi = min(math.ceil(turn(sc["slow"])), dims - 1)
    out = []
    for i in range(dims // 2):
        ramp = min(max((i - lo) / max(hi - lo, 0.001), 0.0), 1.0)
        out.append(f[i] / sc["factor"] * ramp + f[i] * (1 - ramp))
    return torch.tensor(out, dtype=dtype), 0.1 * math.log(sc["factor"]) + 1.0


def rotate_neighbours(x, positions, rot):
    """x [T, ..., n]: elements 2i and 2i + 1 of the first rot.dims form a pair."""
    if not rot or not rot.get("dims") or x.shape[-1] == 0:
        return x
    dims = rot["dims"]
    freq, amp = blended_frequencies(rot, x.dtype)
    angle = positions.to(x.dtype)[:, None] * freq[None, :]
    shape = [x.shape[0]] + [1] * (x.dim() - 2) + [dims // 2]
    cos, sin = amp * torch.cos(angle).view(shape), amp * torch.sin(angle).view(shape)
    out = x.clone()
    a, b = x[..., 0:dims:2], x[..., 1:dims:2]
    out[..., 0:dims:2] = a * cos - b * sin
    out[..., 1:dims:2] = b * cos + a * sin
    return out


def latent_of(h, w, p, m, eps):
    """What a layer with a down projection of its own caches: (latent [T, rank], rotated key part [T, rot_dim])."""
    R = m["kv_rank"]
    down = h @ w[p + "dkv"].T
    c = rms(down[:, :R], eps) * w[p + "dkv.norm"]
    return c, rotate_neighbours(down[:, R:], torch.arange(h.shape[0]), m.get("rot"))


def latent_attention(h, w, p, m, eps, cached):
    T = h.shape[0]
    H, D, Rd, V = m["heads"], m["dim"], m.get("rot_dim", 0), m["vdim"]
    c, k_rot = cached
    q = (h @ w[p + "q"].T).view(T, H, D + Rd)
    q_plain, q_rot = q[..., :D], rotate_neighbours(q[..., D:], torch.arange(T), m.get("rot"))
    k_plain = (c @ w[p + "uk"].T).view(T, H, D)
    v = (c @ w[p + "uv"].T).view(T, H, V)
    size = m["mask"]["size"] if m.get("mask") else T + 1
    out = torch.zeros(T, H, V, dtype=h.dtype)
    for head in range(H):
        for i in range(T):
            lo = max(0, i - size + 1)
            s = (k_plain[lo:i + 1, head] @ q_plain[i, head] + k_rot[lo:i + 1] @ q_rot[i, head]) * m["scale"]
            out[i, head] = torch.softmax(s, 0) @ v[lo:i + 1, head]
    return out.reshape(T, H * V) @ w[p + "o"].T


# ---------------------------------------------------------------------------- feed-forwards
def gated_unit(h, w, p, act):
    return (act(h @ w[p + "gate"].T) * (h @ w[p + "up"].T)) @ w[p + "down"].T


def corrected_experts(h, w, p, f):
    T = h.shape[0]
    top, scale = f["router"]["top"], f["router"]["scale"]
    s = torch.sigmoid(h @ w[p + "router"].T)
    out = torch.zeros(T, h.shape[1], dtype=h.dtype)
    for t in range(T):
        chosen = torch.topk(s[t] + w[p + "correction"], top).indices.tolist()
        total = sum(s[t, e] for e in chosen) + 1e-20
        for e in chosen:
            out[t] = out[t] + s[t, e] / total * scale * gated_unit(h[t], w, f"{p}e{e}.", silu)
    if f.get("shared"):
        out = out + gated_unit(h, w, p + "shared.", silu)
    return out


# ---------------------------------------------------------------------------- the model
def forward(cfg, w, tokens, dtype=F, streams=None):
    """Logits [T, vocab] of one whole sequence. `streams`: a list that receives the stream after every layer."""
    w = {k: v.to(dtype) for k, v in w.items()}
    eps, mult = cfg["norm"]["eps"], cfg.get("residual_mult", 1.0)
    x = w["embed"][torch.as_tensor(tokens, dtype=torch.long)] * (cfg.get("embedding") or {}).get("scale", 1.0)
    latents = {}
    for i, layer in enumerate(cfg["layers"]):
        p, m = f"l{i}.", layer["mixer"]
        h = layer_norm(x, w[p + "norm1"], w[p + "norm1.b"], eps)
        if layer["type"] == "channel_delta":
            mixed = channel_delta(h, w, p + "mix.", m, eps)
        elif layer["type"] == "parallel":
            mixed = side_by_side(h, w, p + "mix.", m, eps)
        else:
            if m.get("kv_from") is None:
                latents[i] = latent_of(h, w, p + "mix.", m, eps)
            mixed = latent_attention(h, w, p + "mix.", m, eps, latents[m["kv_from"] if m.get("kv_from") is not None else i])
        f = layer.get("mlp")
        if f is not None:
            mixed = mixed + (gated_unit(h, w, p + "mlp.", torch.relu) if f["kind"] == "dense" else corrected_experts(h, w, p + "mlp.", f))
        x = x + mult * mixed
        if streams is not None:
            streams.append(x)
    return layer_norm(x, w["final.norm"], w["final.norm.b"], eps) @ w["head"].T
