"""A plain, slow implementation of the Sezanex decoder: one function per mechanism, whole sequences at once,
float64 unless told otherwise. It shares no code with the package; the tests compare the engine with it.

A model is (config dictionary, {tensor name: tensor}). Weights are [out, in] and applied as W x.

    embedding:   x = E[token]
    layer:       x = x + dyt_1b(mixer(dyt_1(x)));  x = x + dyt_2b(ff(dyt_2(x)))      (the second line only with a feed-forward)
    dyt:         tanh(alpha x) * w + b, alpha one number
    loop:        layers start .. stop-1 run `times` times with the same weights and a state of their own per pass;
                 before every pass (the first too) x = W_in [x ; x0], x0 the embedding's output
    output:      logits = E dyt_final(x)
"""

import math

import torch

F = torch.float64


def rms(x, eps):
    return x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps)


def silu(z):
    return z * torch.sigmoid(z)


def gelu_erf(z):
    return 0.5 * z * (1 + torch.erf(z / math.sqrt(2.0)))


def softplus(z):
    return torch.where(z > 30, z, torch.log1p(torch.exp(torch.clamp(z, max=30))))


def dyt(x, w, name):
    return torch.tanh(w[name + ".alpha"] * x) * w[name] + w[name + ".b"]


# ---------------------------------------------------------------------------- positions
def yarn_frequencies(rot, dtype=F):
    """The rotation's frequencies and the amplitude of its cosines and sines. Without `scaling`: base^(-2i/dims), 1."""
    dims, base = rot["dims"], rot["base"]
    half = dims // 2
    f = [base ** (-2.0 * i / dims) for i in range(half)]
    sc = rot.get("scaling")
    if not sc:
        return torch.tensor(f, dtype=dtype), 1.0
    factor, original = sc["factor"], sc["original"]

    def turn(t):        # the (fractional) index whose wave turns t times over the original length
        return dims * math.log(original / (2 * math.pi * t)) / (2 * math.log(base))

    lo = max(math.floor(turn(sc["fast"])), 0)
    hi = min(math.ceil(turn(sc["slow"])), dims - 1)
    out = []
    for i in range(half):
        ramp = min(max((i - lo) / max(hi - lo, 0.001), 0.0), 1.0)
        out.append(f[i] / factor * ramp + f[i] * (1 - ramp))
    return torch.tensor(out, dtype=dtype), 0.1 * math.log(factor) + 1.0


def rotate(x, positions, rot):
    """x [T, heads, dim]: element i of the first `dims` is paired with element i + dims/2."""
    if not rot or not rot.get("dims"):
        return x
    dims = rot["dims"]
    half = dims // 2
    freq, amp = yarn_frequencies(rot, x.dtype)
    angle = positions.to(x.dtype)[:, None] * freq[None, :]
    cos, sin = amp * torch.cos(angle)[:, None, :], amp * torch.sin(angle)[:, None, :]
    u, v = x[..., :half], x[..., half:dims]
    return torch.cat([u * cos - v * sin, v * cos + u * sin, x[..., dims:]], -1)


# ---------------------------------------------------------------------------- mixers
def window_attention(h, w, p, m, eps):
    """Grouped-query attention: RMS norm over the whole of q and of k (before the heads are split), partial
    rotation, a window of mask.size positions (itself included), and a one in the softmax's denominator."""
    T = h.shape[0]
    H, G, D, V = m["heads"], m["kv_heads"], m["dim"], m["vdim"]
    q = rms(h @ w[p + "q"].T, eps) * w[p + "q.norm"]
    k = rms(h @ w[p + "k"].T, eps) * w[p + "k.norm"]
    v = (h @ w[p + "v"].T).view(T, G, V)
    pos = torch.arange(T)
    q = rotate(q.view(T, H, D), pos, m.get("rot"))
    k = rotate(k.view(T, G, D), pos, m.get("rot"))
    size = m["mask"]["size"] if m.get("mask") else T + 1
    out = torch.zeros(T, H, V, dtype=h.dtype)
    for head in range(H):
        g = head // (H // G)
        for i in range(T):
            lo = max(0, i - size + 1)
            s = (k[lo:i + 1, g] @ q[i, head]) * m["scale"]
            top = torch.clamp(s.max(), min=0.0)
            e = torch.exp(s - top)
            pr = e / (torch.exp(-top) + e.sum())
            out[i, head] = pr @ v[lo:i + 1, g]
    return out.reshape(T, H * V) @ w[p + "o"].T


def causal_conv_silu(x, weight, bias):
    """x [T, C]; weight [C, taps], the last column is the current token's; zeros before the start."""
    T, C = x.shape
    taps = weight.shape[1]
    padded = torch.cat([torch.zeros(taps - 1, C, dtype=x.dtype), x], 0)
    out = torch.zeros(T, C, dtype=x.dtype)
    for j in range(taps):
        out = out + padded[j:j + T] * weight[:, j]
    return silu(out + bias)


def mamba2_mixer(h, w, p, m, eps):
    """State-space duality: per head a matrix state S [N, vdim], S_t = exp(-exp(A_log) dt_t) S_(t-1) + dt_t B_t x_t^T,
    y_t = S_t^T C_t + D x_t; then y * silu(z), RMS norm in `norm_groups` equal parts, W_o."""
    T = h.shape[0]
    H, P, N, G, R = m["heads"], m["vdim"], m["state"], m["groups"], m["norm_groups"]
    inner = H * P
    proj = h @ w[p + "in"].T
    z, xbc, dt = proj[:, :inner], proj[:, inner:2 * inner + 2 * G * N], proj[:, 2 * inner + 2 * G * N:]
    xbc = causal_conv_silu(xbc, w[p + "conv"], w[p + "conv.b"])
    x = xbc[:, :inner].view(T, H, P)
    B = xbc[:, inner:inner + G * N].view(T, G, N)
    C = xbc[:, inner + G * N:].view(T, G, N)
    dt = softplus(dt + w[p + "dt_bias"])
    rate = torch.exp(w[p + "A_log"])
    y = torch.zeros(T, H, P, dtype=h.dtype)
    for head in range(H):
        g = head // (H // G)
        S = torch.zeros(N, P, dtype=h.dtype)
        for t in range(T):
            S = torch.exp(-rate[head] * dt[t, head]) * S + dt[t, head] * torch.outer(B[t, g], x[t, head])
            y[t, head] = S.T @ C[t, g] + w[p + "D"][head] * x[t, head]
    y = y.reshape(T, inner) * silu(z)
    y = rms(y.view(T, R, inner // R), eps).reshape(T, inner) * w[p + "norm"]
    return y @ w[p + "o"].T


# ---------------------------------------------------------------------------- feed-forwards
def dense_ff(h, w, p):
    return gelu_erf(h @ w[p + "up"].T) @ w[p + "down"].T


def sigmoid_experts(h, w, p, f):
    """Scores sigmoid(W_r h); the `top` largest are chosen; a chosen expert's score multiplies its INPUT:
    out = sum_e expert_e(s_e h), expert(u) = W_down (silu(W_gate u) * (W_up u))."""
    T = h.shape[0]
    top = f["router"]["top"]
    s = torch.sigmoid(h @ w[p + "router"].T)
    out = torch.zeros(T, w[p + "e0.down"].shape[0], dtype=h.dtype)
    for t in range(T):
        chosen = torch.topk(s[t], top).indices.tolist()
        for e in chosen:
            u = s[t, e] * h[t]
            out[t] = out[t] + (silu(w[f"{p}e{e}.gate"] @ u) * (w[f"{p}e{e}.up"] @ u)) @ w[f"{p}e{e}.down"].T
    return out


# ---------------------------------------------------------------------------- the model
def layer_order(cfg):
    """[(layer index, first of a pass?)] in the order in which layers run."""
    n = len(cfg["layers"])
    loop = cfg.get("loop")
    if not loop:
        return [(i, False) for i in range(n)]
    order = [(i, False) for i in range(loop["start"])]
    for _ in range(loop["times"]):
        order += [(i, i == loop["start"]) for i in range(loop["start"], loop["stop"])]
    return order + [(i, False) for i in range(loop["stop"], n)]


def forward(cfg, w, tokens, dtype=F, streams=None):
    """Logits [T, vocab] of one whole sequence. `streams`: a list that receives the stream after every layer run."""
    w = {k: v.to(dtype) for k, v in w.items()}
    eps = cfg["norm"]["eps"]
    x = w["embed"][torch.as_tensor(tokens, dtype=torch.long)]
    x0 = x
    for i, enters in layer_order(cfg):
        layer, p = cfg["layers"][i], f"l{i}."
        if enters:
            x = torch.cat([x, x0], -1) @ w["loop.in"].T
        hin = dyt(x, w, p + "norm1")
        if layer["type"] == "attention":
            mixed = window_attention(hin, w, p + "mix.", layer["mixer"], eps)
        else:
            mixed = mamba2_mixer(hin, w, p + "mix.", layer["mixer"], eps)
        x = x + dyt(mixed, w, p + "norm1b")
        f = layer.get("mlp")
        if f is not None:
            hin = dyt(x, w, p + "norm2")
            fed = dense_ff(hin, w, p + "mlp.") if f["kind"] == "dense" else sigmoid_experts(hin, w, p + "mlp.", f)
            x = x + dyt(fed, w, p + "norm2b")
        if streams is not None:
            streams.append(x)
    return dyt(x, w, "final.norm") @ w["embed"].T
