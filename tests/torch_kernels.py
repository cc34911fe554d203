"""Plain PyTorch twins of the engine's kernels, one per kernel, for tests only.

They serve two purposes. On the GPU each hand-written kernel is compared with its twin.
On the CPU the twins stand in for the kernel table, so that the cache manager, the step
function, the scheduler and the parts can be exercised where no GPU is present. They are
slow, use no cache-specific tricks (pages are gathered into dense tensors, one segment at
a time) and are not part of the package.
"""

from __future__ import annotations

import torch


class TorchKernels:
    name = "torch-twin"
    max_top_k = 64

    def __init__(self, device="cpu"):
        self.device = torch.device(device)
        self.launches = 0

    def check_status(self):
        pass

    def attention_tables(self, seg_lens, seg_pos0, rep, fixed_tokens=0):
        return {}            # the twin's attention walks the segments by itself

    # ------------------------------------------------------------------ elementwise
    def embedding(self, table, token_ids, scale=1.0):
        return table[token_ids.long()].to(torch.float32) * scale

    def softcap(self, logits, cap):
        logits.copy_(cap * torch.tanh(logits / cap))
        return logits

    def add_rmsnorm(self, residual, delta, weight, eps, out_dtype):
        if delta is not None:
            residual += delta.to(torch.float32)
        scale = torch.rsqrt(residual.pow(2).mean(dim=-1, keepdim=True) + eps)
        return (residual * scale * weight.to(torch.float32)).to(out_dtype)

    def swiglu(self, gate_up):
        inter = gate_up.shape[1] // 2
        g, u = gate_up[:, :inter].float(), gate_up[:, inter:].float()
        return (g / (1 + torch.exp(-g)) * u).to(gate_up.dtype)

    def gather_rows(self, x, rows):
        return x[rows.long()].clone()

    def linear(self, x, w, out_dtype=None, accumulate=None, next_norm=None):
        # `accumulate` is an offer, not an order: the twin returns the product and the caller adds it
        return (x.float() @ w.float().t()).to(out_dtype or x.dtype)

    def linear_swiglu(self, x, w_gate_up):
        return self.swiglu(self.linear(x, w_gate_up))

    def fused_qkv_rope(self, *args, **kwargs):
        return None          # the twin has no fused form: the caller runs projection, rotation and write one by one

    # ------------------------------------------------------------------ attention
    def rope_kv_write(self, qkv, batch, inv_freq, rotary_dim, heads, kv_heads, head_dim, view, write_kv=True,
                      interleaved=False):
        T = qkv.shape[0]
        x = qkv.view(T, heads + 2 * kv_heads, head_dim)
        n_rot = heads + kv_heads
        if rotary_dim and interleaved:
            angles = batch.positions.to(torch.float32)[:, None] * inv_freq[None, :]
            cos, sin = torch.cos(angles)[:, None, :], torch.sin(angles)[:, None, :]
            a = x[:, :n_rot, 0:rotary_dim:2].float().clone()
            b = x[:, :n_rot, 1:rotary_dim:2].float().clone()
            x[:, :n_rot, 0:rotary_dim:2] = (a * cos - b * sin).to(qkv.dtype)
            x[:, :n_rot, 1:rotary_dim:2] = (b * cos + a * sin).to(qkv.dtype)
        elif rotary_dim:
            half = rotary_dim // 2
            angles = batch.positions.to(torch.float32)[:, None] * inv_freq[None, :]
            cos, sin = torch.cos(angles)[:, None, :], torch.sin(angles)[:, None, :]
            a = x[:, :n_rot, :half].float().clone()
            b = x[:, :n_rot, half:rotary_dim].float().clone()
            x[:, :n_rot, :half] = (a * cos - b * sin).to(qkv.dtype)
            x[:, :n_rot, half:rotary_dim] = (b * cos + a * sin).to(qkv.dtype)
        if not write_kv or view is None:
            return
        P = view.page_size
        pos = batch.positions.long()
        pages = view.block_table[batch.seg_of_token.long(), pos // P].long()
        view.keys[pages, :, pos % P, :] = x[:, heads:heads + kv_heads, :]
        view.values[pages, :, pos % P, :] = x[:, heads + kv_heads:, :]

    def paged_attention(self, qkv, batch, heads, kv_heads, head_dim, scale, view):
        T = qkv.shape[0]
        q_all = qkv.view(T, heads + 2 * kv_heads, head_dim)[:, :heads, :].float()
        out = torch.empty(T, heads, head_dim, dtype=torch.float32, device=qkv.device)
        P = view.page_size
        start = 0
        for r, n in enumerate(batch.seg_lens):
            pos0 = batch.seg_pos0_list[r]
            ctx = pos0 + n
            n_pages = -(-ctx // P)
            pages = view.block_table[r, :n_pages].long()
            k = view.keys[pages].permute(0, 2, 1, 3).reshape(n_pages * P, kv_heads, head_dim)[:ctx].float()
            v = view.values[pages].permute(0, 2, 1, 3).reshape(n_pages * P, kv_heads, head_dim)[:ctx].float()
            rep = heads // kv_heads
            k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
            q = q_all[start:start + n]
            scores = torch.einsum("thd,shd->hts", q, k) * scale
            qpos = torch.arange(pos0, ctx, device=qkv.device)[:, None]
            kpos = torch.arange(ctx, device=qkv.device)[None, :]
            visible = kpos <= qpos
            if view.window:
                visible &= kpos > qpos - view.window
            scores = scores.masked_fill(~visible[None], float("-inf"))
            out[start:start + n] = torch.einsum("hts,shd->thd", torch.softmax(scores, dim=-1), v)
            start += n
        return out.reshape(T, heads * head_dim).to(qkv.dtype)

    # ------------------------------------------------------------------ layer norm around sub-layers
    @staticmethod
    def _layernorm(x, norm):
        mean = x.mean(dim=-1, keepdim=True)
        dev = x - mean
        y = dev * torch.rsqrt((dev * dev).mean(dim=-1, keepdim=True) + norm.eps) * norm.weight
        return y + norm.bias if norm.bias is not None else y

    def add_layernorm(self, residual, delta, after, mult, norm, out_dtype):
        if delta is not None:
            d = delta.to(torch.float32)
            residual += mult * (self._layernorm(d, after) if after is not None else d)
        if norm is None:
            return None
        return self._layernorm(residual, norm).to(out_dtype)

    def add_layernorm_sum(self, residual, tensors, scales, row_term, norm, out_dtype):
        for i, t in enumerate(tensors):
            residual += t.to(torch.float32) * (1.0 if scales is None else scales[i])
        if row_term is not None:
            residual += row_term[0] * row_term[1]
        if norm is None:
            return None
        return self._layernorm(residual, norm).to(out_dtype)

    def add_row_vector(self, x, vector):
        x.copy_((x.float() + vector).to(x.dtype))
        return x

    # ------------------------------------------------------------------ latent attention
    @staticmethod
    def _rotate(x, positions, inv_freq, rotary_dim):
        """x [T, ..., D] float32: pairs (i, i + rotary_dim/2) of the first rotary_dim elements."""
        half = rotary_dim // 2
        angles = positions.to(torch.float32)[:, None] * inv_freq[None, :]
        shape = [x.shape[0]] + [1] * (x.dim() - 2) + [half]
        cos, sin = torch.cos(angles).view(shape), torch.sin(angles).view(shape)
        out = x.clone()
        a, b = x[..., :half], x[..., half:rotary_dim]
        out[..., :half] = a * cos - b * sin
        out[..., half:rotary_dim] = b * cos + a * sin
        return out

    def latent_prepare(self, down, batch, q_rank, kv_rank, rot_dim, q_norm, kv_norm, eps, inv_freq, rotary_dim, view,
                       write, out_dtype, amplitude=1.0):
        down = down.float()
        cq = None
        if q_rank:
            cq = down[:, :q_rank]
            cq = (cq * torch.rsqrt(cq.pow(2).mean(-1, keepdim=True) + eps) * q_norm).to(out_dtype)
        if not (write and view is not None):
            return cq
        c = down[:, q_rank:q_rank + kv_rank]
        c = c * torch.rsqrt(c.pow(2).mean(-1, keepdim=True) + eps) * kv_norm
        row = c
        if rot_dim:
            raw = down[:, q_rank + kv_rank:q_rank + kv_rank + rot_dim]
            shared = self._rotate(raw, batch.positions, inv_freq, rotary_dim)
            shared[:, :rotary_dim] *= amplitude
            row = torch.cat([c, shared], dim=-1)
        P = view.page_size
        pos = batch.positions.long()
        pages = view.block_table[batch.seg_of_token.long(), pos // P].long()
        view.rows[pages, pos % P] = row.to(view.rows.dtype)
        return cq

    def heads_linear(self, x, w, out_dtype=None):
        """x [T, H, K] (any strides), w [H, N, K] -> [T, H, N]."""
        return torch.einsum("thk,hnk->thn", x.float(), w.float()).to(out_dtype or x.dtype)

    def latent_attention(self, q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, amplitude=1.0, window="view"):
        T, H, R = q_latent.shape
        out = torch.empty(T, H, R, dtype=torch.float32, device=q_latent.device)
        P = view.page_size
        ql = q_latent.float()
        window = view.window if window == "view" else window
        qr = None
        if q_rot is not None:
            qr = self._rotate(q_rot.float(), batch.positions, inv_freq, rotary_dim)
            qr[..., :rotary_dim] *= amplitude
        start = 0
        for r, n in enumerate(batch.seg_lens):
            pos0 = batch.seg_pos0_list[r]
            ctx = pos0 + n
            n_pages = -(-ctx // P)
            rows = view.rows[view.block_table[r, :n_pages].long()].reshape(n_pages * P, -1)[:ctx].float()
            rows = torch.where(torch.isfinite(rows), rows, torch.zeros_like(rows))     # pages behind the window may be anyone's by now
            scores = torch.einsum("thr,sr->hts", ql[start:start + n], rows[:, :R])
            if qr is not None:
                scores = scores + torch.einsum("thd,sd->hts", qr[start:start + n], rows[:, R:])
            scores = scores * scale
            qpos = torch.arange(pos0, ctx, device=ql.device)[:, None]
            kpos = torch.arange(ctx, device=ql.device)[None, :]
            visible = kpos <= qpos
            if window:
                visible = visible & (kpos > qpos - window)
            scores = scores.masked_fill(~visible[None], float("-inf"))
            if sinks is not None:
                full = torch.cat([scores, sinks.view(H, 1, 1).expand(H, n, 1)], dim=-1)
                weights = torch.softmax(full, dim=-1)[..., :ctx]
            else:
                weights = torch.softmax(scores, dim=-1)
            out[start:start + n] = torch.einsum("hts,sr->thr", weights, rows[:, :R])
            start += n
        return out.to(q_latent.dtype)

    def latent_attention_out(self, q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, w_uv, gate, amplitude=1.0,
                             window="view"):
        mixed = self.latent_attention(q_latent, q_rot, batch, view, scale, sinks, inv_freq, rotary_dim, amplitude, window)
        return self.gate_heads(self.heads_linear(mixed, w_uv), gate)

    def gate_heads(self, out, gate):
        T, H, V = out.shape
        o = out.float()
        if gate is not None:
            g = torch.sigmoid(gate.float())
            o = o * (g[:, :, None] if g.shape[1] == H else g.view(T, H, V))
        return o.reshape(T, H * V).to(out.dtype)

    # ------------------------------------------------------------------ routed experts
    def route_top(self, x, w_router, experts, top, shared, scores="softmax"):
        logits = x.float() @ w_router.t()
        order = torch.sort(logits[:, :experts], dim=-1, descending=True, stable=True).indices[:, :top]
        chosen = torch.gather(logits[:, :experts], 1, order)
        weight = torch.softmax(chosen, dim=-1) if scores == "softmax" else torch.sigmoid(chosen)
        gate = torch.sigmoid(logits[:, experts]) if shared else None
        return order.to(torch.int32), weight, gate

    @staticmethod
    def _glu_clamped(gate_up, limit, alpha):
        inter = gate_up.shape[-1] // 2
        if not limit > 0:                      # no clamps and no unit offset: the plain gated unit
            g = gate_up[..., :inter].float()
            return g * torch.sigmoid(alpha * g) * gate_up[..., inter:].float()
        g = gate_up[..., :inter].float().clamp(max=limit)
        u = gate_up[..., inter:].float().clamp(min=-limit, max=limit)
        return g * torch.sigmoid(alpha * g) * (u + 1.0)

    def linear_glu_clamped(self, x, w_gate_up, limit, alpha):
        return self._glu_clamped(self.linear(x, w_gate_up), limit, alpha).to(x.dtype)

    def route_corrected(self, x, w_router, correction, experts, top, scale, floor):
        s = torch.sigmoid(x.float() @ w_router.t())
        order = torch.sort(s + correction, dim=-1, descending=True, stable=True).indices[:, :top]
        chosen = torch.gather(s, 1, order)
        return order.to(torch.int32), chosen / (chosen.sum(-1, keepdim=True) + floor) * scale

    def routed_experts(self, x, choice, weight, w_gate_up, w_down, limit, alpha, shared=None, shared_gate=None):
        T, top = choice.shape
        out = torch.zeros(T, w_down.shape[1], dtype=torch.float32, device=x.device)
        for t in range(T):
            for j in range(top):
                e = int(choice[t, j])
                hidden = self._glu_clamped(self.linear(x[t:t + 1], w_gate_up[e]), limit, alpha).to(x.dtype)
                out[t] += weight[t, j] * self.linear(hidden, w_down[e]).float()[0]
        if shared is not None:
            shared_out = self.linear(self.linear_glu_clamped(x, shared[0], shared[2], alpha), shared[1])
            out += shared_out.float() * (shared_gate[:, None] if shared_gate is not None else 1.0)
        return out

    # ------------------------------------------------------------------ the float32 stream, several outputs at once
    def stream_add_norm(self, residual, deltas, row_vector=None, weight=None, eps=0.0, offset=0.0, out_dtype=None):
        for d in deltas:
            if d is not None:
                residual += d.to(torch.float32)
        if row_vector is not None:
            residual += row_vector
        if weight is None:
            return None
        scale = 1.0 / torch.sqrt(residual.pow(2).mean(dim=-1, keepdim=True) + eps)
        return (residual * scale * (offset + weight.to(torch.float32))).to(out_dtype)

    def gated_rmsnorm(self, x, weight, eps, gate, out_dtype):
        scale = 1.0 / torch.sqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
        return (x * scale * weight * torch.sigmoid(gate.float())).to(out_dtype)

    def mean_rmsnorm_pair(self, a, wa, b, wb, eps):
        a, b = a.float(), b.float()
        ka = 1.0 / torch.sqrt(a.pow(2).mean(dim=-1, keepdim=True) + eps)
        kb = 1.0 / torch.sqrt(b.pow(2).mean(dim=-1, keepdim=True) + eps)
        return 0.5 * (a * ka * wa + b * kb * wb)

    @staticmethod
    def _gelu_tanh(z):
        return 0.5 * z * (1 + torch.tanh(0.7978845608028654 * (z + 0.044715 * z ** 3)))

    def glu_activation(self, gate_up, activation):
        inter = gate_up.shape[1] // 2
        g, u = gate_up[:, :inter].float(), gate_up[:, inter:].float()
        act = g * torch.sigmoid(g) if activation == "silu" else (torch.relu(g) if activation == "relu" else self._gelu_tanh(g))
        return (act * u).to(gate_up.dtype)

    def activation(self, x, activation, out_dtype):
        if activation == "gelu_erf":
            z = x.float()
            return (0.5 * z * (1 + torch.erf(z * 0.7071067811865476))).to(out_dtype)
        assert activation == "relu2"
        return torch.relu(x.float()).pow(2).to(out_dtype)

    # ------------------------------------------------------------------ Dynamic Tanh around sub-layers, pass mixing
    @staticmethod
    def _dyntanh(x, norm):
        return torch.tanh(norm.alpha * x) * norm.weight + norm.bias

    def add_dyntanh(self, residual, delta, after, mult, norm, out_dtype):
        if delta is not None:
            d = delta.to(torch.float32)
            residual += mult * (self._dyntanh(d, after) if after is not None else d)
        if norm is None:
            return None
        return self._dyntanh(residual, norm).to(out_dtype)

    def concat_cast(self, a, b, out_dtype):
        return torch.cat([a, b], 1).to(out_dtype)

    # ------------------------------------------------------------------ experts whose weight multiplies their input
    def input_weighted_experts(self, x, choice, weight, w_gate_up, w_down):
        T, top = choice.shape
        inter = w_gate_up.shape[1] // 2
        out = torch.zeros(T, w_down.shape[1], dtype=torch.float32, device=x.device)
        for t in range(T):
            for j in range(top):
                e = int(choice[t, j])
                u = (x[t:t + 1].float() * weight[t, j]).to(x.dtype)
                gu = self.linear(u, w_gate_up[e], out_dtype=torch.float32)
                g = gu[:, :inter]
                hidden = (g * torch.sigmoid(g) * gu[:, inter:]).to(x.dtype)
                out[t] += self.linear(hidden, w_down[e]).float()[0]
        return out

    # ------------------------------------------------------------------ state-space mixer
    def state_space(self, proj, conv_w, conv_b, dt_bias, rate, skip, norm_w, eps, heads, vdim, state, groups, norm_groups,
                    batch, view, write_state=True):
        T = proj.shape[0]
        inner, GN = heads * vdim, groups * state
        C, taps = inner + 2 * GN, conv_w.shape[1]
        z = proj[:, :inner].float()
        xin = proj[:, inner:inner + C]
        dt = torch.nn.functional.softplus(proj[:, inner + C:inner + C + heads].float() + dt_bias, threshold=30.0)
        decay = torch.exp(-rate * dt)
        y = torch.empty(T, heads, vdim, dtype=torch.float32, device=proj.device)
        start, keep = 0, taps - 1
        for n, slot in zip(batch.seg_lens, batch.seg_slot_list):
            kept = view.tail[slot][:keep] if keep > 0 else xin[:0]
            seq = torch.cat([kept.to(xin.dtype), xin[start:start + n]], 0)
            acc = conv_b[None, :].repeat(n, 1)
            for j in range(taps):
                acc = acc + seq[j:j + n].float() * conv_w[:, j]
            u = (acc * torch.sigmoid(acc)).to(proj.dtype).float()
            xs = u[:, :inner].view(n, heads, vdim)
            B = u[:, inner:inner + GN].view(n, groups, state).repeat_interleave(heads // groups, dim=1)
            Cm = u[:, inner + GN:].view(n, groups, state).repeat_interleave(heads // groups, dim=1)
            S = view.state[slot].clone()
            for i in range(n):
                t = start + i
                S = decay[t][:, None, None] * S + (dt[t][:, None] * B[i])[:, :, None] * xs[i][:, None, :]
                y[t] = torch.einsum("hnp,hn->hp", S, Cm[i]) + skip[:, None] * xs[i]
            if write_state:
                view.state[slot] = S
                if keep > 0:
                    view.tail[slot][:keep] = seq[-keep:]
            start += n
        gated = y.reshape(T, inner) * (z * torch.sigmoid(z))
        parts = gated.view(T, norm_groups, inner // norm_groups)
        normed = parts * torch.rsqrt(parts.pow(2).mean(-1, keepdim=True) + eps)
        return (normed.reshape(T, inner) * norm_w).to(proj.dtype)

    # ------------------------------------------------------------------ recurrent mixers
    def lightning_attention(self, proj, batch, view, heads, dim, vdim, decays, write_state=True):
        T = proj.shape[0]
        act = proj.float()
        act = act * torch.sigmoid(act)
        q = act[:, :heads * dim].view(T, heads, dim)
        k = act[:, heads * dim:2 * heads * dim].view(T, heads, dim)
        v = act[:, 2 * heads * dim:2 * heads * dim + heads * vdim].view(T, heads, vdim)
        out = torch.empty(T, heads, vdim, dtype=torch.float32, device=proj.device)
        start = 0
        for r, n in enumerate(batch.seg_lens):
            slot = batch.seg_slot_list[r]
            S = view.state[slot].clone()
            for t in range(start, start + n):
                S = decays[:, None, None] * S + k[t][:, :, None] * v[t][:, None, :]
                out[t] = torch.einsum("hdv,hd->hv", S, q[t])
            if write_state:
                view.state[slot] = S
            start += n
        return out.reshape(T, heads * vdim)

    def causal_conv(self, x, bias_x, conv_w, conv_b, batch, view):
        T, C = x.shape
        taps = conv_w.shape[1]
        xin = (x.float() + bias_x).to(x.dtype).float()
        u = torch.empty(T, C, dtype=torch.float32, device=x.device)
        start = 0
        for r, n in enumerate(batch.seg_lens):
            slot = batch.seg_slot_list[r]
            kept = view.tail[slot][:taps - 1].float() if taps > 1 else xin[:0]
            seq = torch.cat([kept, xin[start:start + n]], 0)
            acc = conv_b[None, :].repeat(n, 1)
            for j in range(taps):
                acc = acc + seq[j:j + n] * conv_w[:, j]
            u[start:start + n] = acc
            start += n
        return u.to(x.dtype)

    def gated_recurrence(self, u, gates, gate_bias, rate, yx, bias_yx, batch, view, write_state=True):
        T, C = u.shape
        B = gates.shape[1]
        s = C // B
        pre = gates + gate_bias
        r = torch.sigmoid(pre[:, :, :s]).reshape(T, C)
        i = torch.sigmoid(pre[:, :, s:]).reshape(T, C)
        a = torch.exp(-rate * r)
        drive = torch.sqrt((1 - a * a).clamp(min=0)) * (i * u.float())
        y = self._gelu_tanh(yx[:, :C].float() + bias_yx[:C])
        xin = (yx[:, C:].float() + bias_yx[C:]).to(u.dtype)
        out = torch.empty(T, C, dtype=torch.float32, device=u.device)
        start = 0
        keep = view.taps - 1
        for n, slot in zip(batch.seg_lens, batch.seg_slot_list):
            S = view.state[slot].clone()
            for t in range(start, start + n):
                S = a[t] * S + drive[t]
                out[t] = S * y[t]
            if write_state:
                view.state[slot] = S
                if keep > 0:
                    view.tail[slot][:keep] = torch.cat([view.tail[slot][:keep], xin[start:start + n]], 0)[-keep:]
            start += n
        return out.to(u.dtype)

    def recurrent_token(self, yx, bias_yx, conv_w, conv_b, w_gates, gate_bias, rate, batch, view, write_state=True):
        C, B = yx.shape[1] // 2, w_gates.shape[0]
        u = self.causal_conv(yx[:, C:], bias_yx[C:], conv_w, conv_b, batch, view)
        gates = self.heads_linear(u.view(-1, B, C // B), w_gates, out_dtype=torch.float32)
        return self.gated_recurrence(u, gates, gate_bias, rate, yx, bias_yx, batch, view, write_state)

    # ------------------------------------------------------------------ token shift, low-rank maps, matrix states
    def token_shift(self, x, mu, batch, view):
        T, width = x.shape
        out = torch.empty(T, mu.shape[0], width, dtype=torch.float32, device=x.device)
        xf = x.float()
        start = 0
        for n, slot in zip(batch.seg_lens, batch.seg_slot_list):
            before = torch.cat([view.tail[slot][:1].float(), xf[start:start + n - 1]], 0)
            cur = xf[start:start + n]
            out[start:start + n] = cur[:, None, :] + (before - cur)[:, None, :] * mu[None]
            start += n
        return out.to(x.dtype)

    def lowrank_expand(self, x, w, bias, in_act, out_kind, rate=None):
        z = x.float()
        if in_act == "tanh":
            z = torch.tanh(z)
        z = z @ w.float().t()
        if bias is not None:
            z = z + bias
        if out_kind == "neg_exp":
            return -torch.exp(z)
        if out_kind == "neg_rate_softplus":
            heads = rate.shape[0]
            sp = torch.nn.functional.softplus(z, threshold=30.0)
            return -(sp.view(z.shape[0], heads, -1) * rate[None, :, None]).reshape(z.shape)
        assert out_kind == "none"
        return z

    def shifted_state(self, rkvg, log_decay, bonus, norm_w, eps, heads, dim, x, batch, view, write_state=True):
        four = [rkvg[:, i] for i in range(4)] if torch.is_tensor(rkvg) else list(rkvg)
        T = four[0].shape[0]
        r, k, v = (four[i].float().reshape(T, heads, dim) for i in range(3))
        g = four[3].float()
        w = torch.exp(log_decay).view(T, heads, dim)
        out = torch.empty(T, heads, dim, dtype=torch.float32, device=x.device)
        start = 0
        for n, slot in zip(batch.seg_lens, batch.seg_slot_list):
            S = view.state[slot].clone()
            for t in range(start, start + n):
                kv = k[t][:, :, None] * v[t][:, None, :]
                out[t] = torch.einsum("hkv,hk->hv", S + bonus[:, :, None] * kv, r[t])
                S = w[t][:, :, None] * S + kv
            if write_state:
                view.state[slot] = S
                view.tail[slot][0] = x[start + n - 1]
            start += n
        out = out * torch.rsqrt(out.pow(2).mean(-1, keepdim=True) + eps)
        return (out.reshape(T, heads * dim) * norm_w * (g * torch.sigmoid(g))).to(x.dtype)

    def short_conv_silu(self, x, conv_w, batch, view):
        T, C = x.shape
        taps = conv_w.shape[1]
        out = torch.empty(T, C, dtype=torch.float32, device=x.device)
        start = 0
        for n, slot in zip(batch.seg_lens, batch.seg_slot_list):
            kept = view.tail[slot][:taps - 1].float() if taps > 1 else x[:0].float()
            seq = torch.cat([kept, x[start:start + n].float()], 0)
            acc = torch.zeros(n, C, dtype=torch.float32, device=x.device)
            for j in range(taps):
                acc = acc + seq[j:j + n] * conv_w[:, j]
            out[start:start + n] = acc * torch.sigmoid(acc)
            start += n
        return out.to(x.dtype)

    def delta_rule(self, u, raw, beta, log_decay, gate, norm_w, eps, heads, kv_heads, dim, vdim, batch, view, write_state=True):
        T = u.shape[0]
        qk = kv_heads * dim
        uf = u.float()
        q, k = uf[:, :qk].view(T, kv_heads, dim), uf[:, qk:2 * qk].view(T, kv_heads, dim)
        v = uf[:, 2 * qk:].view(T, heads, vdim)
        q = q / torch.sqrt(q.pow(2).sum(-1, keepdim=True) + 1e-6) * dim ** -0.5
        k = k / torch.sqrt(k.pow(2).sum(-1, keepdim=True) + 1e-6)
        rep = heads // kv_heads
        q, k = q.repeat_interleave(rep, dim=1), k.repeat_interleave(rep, dim=1)
        b = torch.sigmoid(beta.float())
        g = torch.exp(log_decay).view(T, heads, dim)
        out = torch.empty(T, heads, vdim, dtype=torch.float32, device=u.device)
        keep = view.taps - 1
        start = 0
        for n, slot in zip(batch.seg_lens, batch.seg_slot_list):
            S = view.state[slot].clone()
            for t in range(start, start + n):
                S = g[t][:, :, None] * S
                d = b[t][:, None] * (v[t] - torch.einsum("hkv,hk->hv", S, k[t]))
                S = S + k[t][:, :, None] * d[:, None, :]
                out[t] = torch.einsum("hkv,hk->hv", S, q[t])
            if write_state:
                view.state[slot] = S
                if keep > 0:
                    view.tail[slot][:keep] = torch.cat([view.tail[slot][:keep], raw[start:start + n].to(view.tail.dtype)], 0)[-keep:]
            start += n
        out = out * torch.rsqrt(out.pow(2).mean(-1, keepdim=True) + eps) * norm_w
        return (out.reshape(T, heads * vdim) * torch.sigmoid(gate.float())).to(u.dtype)

    # ------------------------------------------------------------------ attention with a sink, a cap, chunks
    def qk_norm_rope_write(self, qkv, batch, q_norm, k_norm, eps, inv_freq, rotary_dim, heads, kv_heads, dim, vdim, view,
                           write_kv=True, whole=False, amplitude=1.0, bias=None, q_temp=None):
        T = qkv.shape[0]
        n_qk = heads + kv_heads
        if bias is not None:
            qkv.copy_((qkv.float() + bias).to(qkv.dtype))
        x = qkv[:, :n_qk * dim].float().clone().view(T, n_qk, dim)
        if q_norm is not None and whole:
            q, k = x[:, :heads].reshape(T, -1), x[:, heads:].reshape(T, -1)
            q = q / torch.sqrt(q.pow(2).mean(-1, keepdim=True) + eps) * q_norm
            k = k / torch.sqrt(k.pow(2).mean(-1, keepdim=True) + eps) * k_norm
            x = torch.cat([q.view(T, heads, dim), k.view(T, kv_heads, dim)], 1)
        elif q_norm is not None:
            x = x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + eps)
            x = torch.cat([x[:, :heads] * q_norm, x[:, heads:] * k_norm], 1)
        if q_temp is not None:
            runs = torch.div(batch.positions + 1, q_temp[1], rounding_mode="floor").to(torch.float32)
            x[:, :heads] = x[:, :heads] * (1.0 + q_temp[0] * torch.log(runs + 1.0))[:, None, None]
        if rotary_dim:
            half = rotary_dim // 2
            angles = batch.positions.to(torch.float32)[:, None] * inv_freq[None, :]
            cos, sin = amplitude * torch.cos(angles)[:, None, :], amplitude * torch.sin(angles)[:, None, :]
            a, b = x[..., :half], x[..., half:rotary_dim]
            x = torch.cat([a * cos - b * sin, b * cos + a * sin, x[..., rotary_dim:]], -1)
        qkv[:, :n_qk * dim] = x.reshape(T, n_qk * dim).to(qkv.dtype)
        if not write_kv or view is None:
            return
        P = view.page_size
        pos = batch.positions.long()
        pages = view.block_table[batch.seg_of_token.long(), pos // P].long()
        view.keys[pages, :, pos % P, :] = qkv[:, heads * dim:n_qk * dim].view(T, kv_heads, dim)
        view.values[pages, :, pos % P, :] = qkv[:, n_qk * dim:].view(T, kv_heads, vdim)

    def sink_attention(self, qkv, batch, heads, kv_heads, dim, vdim, scale, softcap, sinks, view, distance_bias=None):
        T = qkv.shape[0]
        q_all = qkv[:, :heads * dim].float().view(T, heads, dim)
        out = torch.empty(T, heads, vdim, dtype=torch.float32, device=qkv.device)
        P = view.page_size
        start = 0
        for r, n in enumerate(batch.seg_lens):
            pos0 = batch.seg_pos0_list[r]
            ctx = pos0 + n
            n_pages = -(-ctx // P)
            pages = view.block_table[r, :n_pages].long()
            k = view.keys[pages].permute(0, 2, 1, 3).reshape(n_pages * P, kv_heads, dim)[:ctx].float()
            v = view.values[pages].permute(0, 2, 1, 3).reshape(n_pages * P, kv_heads, vdim)[:ctx].float()
            rep = heads // kv_heads
            k, v = k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1)
            scores = torch.einsum("thd,shd->hts", q_all[start:start + n], k) * scale
            if softcap:
                scores = softcap * torch.tanh(scores / softcap)
            qpos = torch.arange(pos0, ctx, device=qkv.device)[:, None]
            kpos = torch.arange(ctx, device=qkv.device)[None, :]
            if distance_bias is not None:
                far = distance_bias.shape[1] - 1
                scores = scores + distance_bias[:, (qpos - kpos).clamp(0, far)]
            visible = kpos <= qpos
            if view.window:
                visible &= kpos > qpos - view.window
            if view.chunk:
                visible &= (kpos // view.chunk) == (qpos // view.chunk)
            scores = scores.masked_fill(~visible[None], float("-inf"))
            if sinks is not None:
                scores = torch.cat([scores, sinks[:, None, None].expand(heads, n, 1)], -1)
            weights = torch.softmax(scores, dim=-1)[..., :ctx]
            # pages that a chunk or a window has passed may have been given back: what they hold now has weight 0
            v = torch.where(torch.isfinite(v), v, torch.zeros_like(v))
            out[start:start + n] = torch.einsum("hts,shd->thd", weights, v)
            start += n
        return out.reshape(T, heads * vdim).to(qkv.dtype)

    # ------------------------------------------------------------------ experts chosen from the best groups
    def route_grouped(self, x, w_router, experts, top, groups, keep, floor):
        s = torch.softmax(x.float() @ w_router.t(), dim=-1)
        T = s.shape[0]
        per = experts // groups
        best = s.view(T, groups, per).max(-1).values
        kept = torch.sort(best, dim=-1, descending=True, stable=True).indices[:, :keep]
        allowed = torch.zeros(T, groups, dtype=torch.bool, device=x.device)
        allowed.scatter_(1, kept, True)
        masked = torch.where(allowed.repeat_interleave(per, 1), s, torch.full_like(s, -1.0))
        order = torch.sort(masked, dim=-1, descending=True, stable=True).indices[:, :top]
        chosen = torch.gather(s, 1, order)
        return order.to(torch.int32), chosen / (chosen.sum(-1, keepdim=True) + floor)

    def plain_experts(self, x, choice, weight, w_up, w_down, activation="relu2"):
        T, top = choice.shape
        out = torch.zeros(T, w_down.shape[1], dtype=torch.float32, device=x.device)
        for t in range(T):
            for j in range(top):
                e = int(choice[t, j])
                hidden = self.activation(self.linear(x[t:t + 1], w_up[e], out_dtype=torch.float32), activation, x.dtype)
                out[t] += weight[t, j] * self.linear(hidden, w_down[e]).float()[0]
        return out

    # ------------------------------------------------------------------ sampling
    @staticmethod
    def uniform(seed: int, counter: int) -> float:
        """u in [0, 1) from (seed, counter): a 64-bit mix, top 24 bits."""
        mask = (1 << 64) - 1
        x = (seed & mask) ^ ((counter + 0x9E3779B97F4A7C15) & mask)
        x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & mask
        x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & mask
        x ^= x >> 31
        return (x >> 40) / 16777216.0

    def sample(self, logits, temperature=None, top_k=None, top_p=None, seeds=None, counters=None):
        rows, vocab = logits.shape
        out = torch.empty(rows, dtype=torch.int32, device=logits.device)
        for r in range(rows):
            l = logits[r].float().cpu()
            best = int(torch.argmax(l))          # torch.argmax gives the first of equal maxima on the CPU
            temp = float(temperature[r]) if temperature is not None else 0.0
            if not temp > 0:
                out[r] = best
                continue
            u = self.uniform(int(seeds[r]), int(counters[r]))
            k = int(top_k[r]) if top_k is not None else 0
            p_limit = float(top_p[r]) if top_p is not None else 1.0
            probs = torch.exp((l - l[best]) / temp)
            if k <= 0 or k > self.max_top_k:
                # cuts as thresholds on the value: below the k-th largest logit, then the low tail that holds at
                # most 1 - top_p of what is left; logits equal to a threshold stay; the draw walks the ids in order
                keep = torch.ones(vocab, dtype=torch.bool)
                if 0 < k < vocab:
                    keep &= l >= torch.sort(l, descending=True).values[k - 1]
                if p_limit < 1.0:
                    masked = torch.where(keep, probs.double(), torch.zeros((), dtype=torch.float64))
                    limit = (1.0 - p_limit) * float(masked.sum())
                    values, order = torch.sort(l)                        # ascending
                    mass = torch.cumsum(masked[order], 0)
                    first = torch.searchsorted(values, values, right=False)   # where each value's equals begin
                    below = torch.where(first > 0, mass[(first - 1).clamp(min=0)], torch.zeros((), dtype=torch.float64))
                    fits = (below <= limit) & keep[order]
                    t = values[int(fits.nonzero().max())]                # the largest value whose lower tail fits
                    keep &= l >= torch.minimum(t, l[best])
                probs = torch.where(keep, probs, torch.zeros(()))
                cdf = torch.cumsum(probs.double(), 0)
                target = u * float(cdf[-1])
                pick = int(torch.searchsorted(cdf, torch.tensor(target, dtype=torch.float64), right=True))
                out[r] = min(pick, vocab - 1)
                continue
            k = min(k, vocab)
            order = sorted(range(vocab), key=lambda i: (-float(l[i]), i))[:k]
            cand = probs[order].double()
            keep = k
            if p_limit < 1.0:
                tail = 0.0
                for c in range(k - 1, 0, -1):
                    tail += float(cand[c] / cand.sum())
                    if tail <= 1.0 - p_limit:
                        keep = c
                    else:
                        break
            cdf = torch.cumsum(cand[:keep], 0)
            target = u * float(cdf[-1])
            pick = int(torch.searchsorted(cdf, torch.tensor(target, dtype=torch.float64), right=True))
            out[r] = order[min(pick, keep - 1)]
        return out
