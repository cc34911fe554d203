"""Bufolorn on the GPU: every kernel of the design against its plain twin, and the whole engine (step function, cache
manager, captured steps, scheduler and entry point) against the plain implementation, in both precisions."""

from types import SimpleNamespace

import pytest
import torch

import bufolorn_cases as cases
import helpers
import plain_bufolorn
from test_bufolorn import (check_a_far_row_of_the_distance_table, check_one_latent_key_inside_the_window_only,
                           check_the_bonus_is_for_the_current_token_only, check_the_matrix_states_keep_a_far_token)
from test_gpu_pedazen import _attention_setup, _batch, _close
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.engine.step import build_engine
from tt_transformers_b200.parts import PagedKV
from tt_transformers_b200.parts.base import LatentPages, MatrixState

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TOL = {torch.float32: 2e-5, torch.bfloat16: 2e-2}


@pytest.fixture(scope="module")
def kernels():
    from tt_transformers_b200.kernels import load_kernels
    return load_kernels(torch.device(DEV))


@pytest.fixture(scope="module")
def twin():
    return TorchKernels(DEV)


# ---------------------------------------------------------------------------- the stream, the norm, small kernels
@pytest.mark.parametrize("width", [60, 128, 1001, 4096])
def test_layer_norm_over_a_weighted_sum(kernels, twin, width):
    g = torch.Generator().manual_seed(width)
    norm = SimpleNamespace(weight=(1 + 0.3 * torch.randn(width, generator=g)).to(DEV), bias=(0.3 * torch.randn(width, generator=g)).to(DEV),
                           eps=1e-5)
    row = torch.randn(width, generator=g).to(DEV)
    for dtypes, scales, row_term, use_norm in (([torch.bfloat16, torch.float32, torch.bfloat16], [0.3, 0.2, 0.5], (row, 0.3), True),
                                               ([torch.float32], None, None, True), ([], None, None, True),
                                               ([torch.bfloat16] * 5, [1.0, 2.0, 3.0, -1.0, 0.5], (row, 1.0), True),
                                               ([torch.float32, torch.float32], [0.5, 0.5], (row, -2.0), False)):
        x = (2 * torch.randn(5, width, generator=g)).to(DEV)
        terms = [torch.randn(5, width, generator=g).to(DEV, dt) for dt in dtypes]
        for out_dtype in (torch.float32, torch.bfloat16):
            x_ref, x_got = x.clone(), x.clone()
            ref = twin.add_layernorm_sum(x_ref, terms, scales, row_term, norm if use_norm else None, out_dtype)
            got = kernels.add_layernorm_sum(x_got, terms, scales, row_term, norm if use_norm else None, out_dtype)
            _close(x_got, x_ref, 2e-6)
            if use_norm:
                _close(got, ref, TOL[out_dtype])
            else:
                assert got is None
    for dtype in (torch.float32, torch.bfloat16):
        wide = torch.randn(7, width + 8, generator=g).to(DEV, dtype)
        a, b = wide.clone(), wide.clone()
        twin.add_row_vector(a[:, :width], row)
        kernels.add_row_vector(b[:, :width], row)
        _close(b, a, TOL[dtype])
        gu = (2 * torch.randn(7, 2 * width, generator=g)).to(DEV, dtype)
        _close(kernels.glu_activation(gu, "relu"), twin.glu_activation(gu, "relu"), TOL[dtype])


@pytest.mark.parametrize("T,rank,N,heads", [(70, 16, 384, 6), (3, 1, 10, 5), (9, 24, 192, 1), (300, 7, 63, 9), (1, 64, 2048, 16)])
def test_low_rank_maps_and_token_shift(kernels, twin, T, rank, N, heads):
    g = torch.Generator().manual_seed(T + N)
    wide = torch.randn(T, rank + 5, generator=g).to(DEV)
    x = wide[:, 3:3 + rank]
    bias, rate = torch.randn(N, generator=g).to(DEV), (3 * torch.rand(heads, generator=g)).to(DEV)
    for dtype in (torch.float32, torch.bfloat16):
        w = (torch.randn(N, rank, generator=g) * rank ** -0.5).to(DEV, dtype)
        for args in ((bias, "tanh", "neg_exp"), (None, None, "none"), (bias, None, "none")):
            _close(kernels.lowrank_expand(x, w, *args), twin.lowrank_expand(x, w, *args), 2e-5)
        if N % heads == 0:
            _close(kernels.lowrank_expand(x, w, bias, None, "neg_rate_softplus", rate=rate),
                   twin.lowrank_expand(x, w, bias, None, "neg_rate_softplus", rate=rate), 2e-5)
    segs, slots = [(0, 23), (40, 1), (7, 2), (0, 1), (64, 50)], [2, 0, 5, 1, 3]
    batch = _batch(segs, slots)
    width = N
    mu = torch.rand(5, width, generator=g).to(DEV)
    for dtype in (torch.float32, torch.bfloat16):
        h = torch.randn(batch.num_tokens, width + 8, generator=g).to(DEV, dtype)[:, :width]
        tail = torch.randn(7, 1, width, generator=g).to(DEV, dtype)
        view = MatrixState(1, 2, 2, width, 2).view({"state": torch.zeros(7, 1, 2, 2, device=DEV), "tail": tail},
                                                   slots=batch.seg_slot, slot_list=slots)
        _close(kernels.token_shift(h, mu, batch, view), twin.token_shift(h, mu, batch, view), TOL[dtype])


# ---------------------------------------------------------------------------- the matrix states
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,D,width", [(2, 32, 96), (1, 5, 7), (3, 7, 60), (2, 64, 128), (4, 24, 50), (1, 128, 130), (2, 200, 64)])
def test_shifted_state_against_its_twin(kernels, twin, dtype, H, D, width):
    """Portions beside single tokens, continuing from a state that is not zero, on slots in any order; a second step
    continues from what the first left; a state that must only be read stays as it was."""
    g = torch.Generator().manual_seed(H * D + width)
    segs, slots = [(0, 37), (90, 1), (5, 2), (0, 1), (300, 70), (0, 17)], [3, 0, 5, 1, 4, 6]
    req = MatrixState(H, D, D, width, 2)
    state = (torch.randn(8, H, D, D, generator=g) * 0.5).to(DEV)
    tail = torch.randn(8, 1, width, generator=g).to(DEV, dtype)
    bonus, norm_w = torch.randn(H, D, generator=g).to(DEV), (1 + 0.3 * torch.randn(H * D, generator=g)).to(DEV)
    for step in range(2):
        batch = _batch(segs, slots)
        T = batch.num_tokens
        rkvg = (torch.randn(T, 4, H * D + 8, generator=g) * D ** -0.25).to(DEV, dtype)[:, :, :H * D]
        log_decay = -torch.exp(torch.randn(T, H * D, generator=g) * 1.5 - 1.5).to(DEV)
        x = torch.randn(T, width, generator=g).to(DEV, dtype)
        s_ref, s_got, t_ref, t_got = state.clone(), state.clone(), tail.clone(), tail.clone()
        v_ref = req.view({"state": s_ref, "tail": t_ref}, slots=batch.seg_slot, slot_list=slots)
        v_got = req.view({"state": s_got, "tail": t_got}, slots=batch.seg_slot, slot_list=slots)
        ref = twin.shifted_state(rkvg, log_decay, bonus, norm_w, 1e-5, H, D, x, batch, v_ref)
        got = kernels.shifted_state(rkvg, log_decay, bonus, norm_w, 1e-5, H, D, x, batch, v_got)
        _close(got, ref, 1e-4 if dtype == torch.float32 else 2e-2)
        _close(s_got, s_ref, 5e-5)
        assert torch.equal(t_got, t_ref)
        assert torch.equal(s_got[[2, 7]], state[[2, 7]]) and torch.equal(t_got[[2, 7]], tail[[2, 7]])       # nobody's slots are nobody's
        kept_s, kept_t = s_got.clone(), t_got.clone()
        kernels.shifted_state(rkvg, log_decay, bonus, norm_w, 1e-5, H, D, x, batch, v_got, write_state=False)
        assert torch.equal(s_got, kept_s) and torch.equal(t_got, kept_t)
        state, tail = s_got, t_got


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,G,D,V,taps", [(4, 2, 16, 24, 4), (1, 1, 6, 10, 1), (6, 2, 3, 7, 2), (2, 1, 64, 64, 3), (4, 4, 128, 32, 4),
                                          (3, 3, 40, 136, 9), (2, 1, 200, 16, 2)])
def test_convolutions_and_delta_rule_against_their_twins(kernels, twin, dtype, H, G, D, V, taps):
    """Portions shorter and longer than the convolutions' reach, single tokens, first tokens; two steps in a row."""
    g = torch.Generator().manual_seed(H * D + V + taps)
    segs, slots = [(0, 23), (40, 1), (7, 2), (0, 1), (11, 3), (64, 50)], [2, 0, 5, 1, 6, 3]
    C = 2 * G * D + H * V
    req = MatrixState(H, D, V, C, taps)
    state = (torch.randn(8, H, D, V, generator=g) * 0.5).to(DEV)
    tail = torch.randn(8, max(taps - 1, 1), C, generator=g).to(DEV, dtype)
    conv_w = (torch.randn(C, taps, generator=g) * 0.5).to(DEV)
    norm_w = (1 + 0.3 * torch.randn(V, generator=g)).to(DEV)
    for step in range(2):
        batch = _batch(segs, slots)
        T = batch.num_tokens
        raw = torch.randn(T, C + 8, generator=g).to(DEV, dtype)[:, :C]
        small = torch.randn(T, H + 5, generator=g).to(DEV)
        log_decay = -(torch.rand(T, H * D, generator=g) * 2).to(DEV)
        gate = torch.randn(T, H * V, generator=g).to(DEV)
        s_ref, s_got, t_ref, t_got = state.clone(), state.clone(), tail.clone(), tail.clone()
        v_ref = req.view({"state": s_ref, "tail": t_ref}, slots=batch.seg_slot, slot_list=slots)
        v_got = req.view({"state": s_got, "tail": t_got}, slots=batch.seg_slot, slot_list=slots)
        u_ref, u_got = twin.short_conv_silu(raw, conv_w, batch, v_ref), kernels.short_conv_silu(raw, conv_w, batch, v_got)
        _close(u_got, u_ref, TOL[dtype])
        ref = twin.delta_rule(u_ref, raw, small[:, 2:2 + H], log_decay, gate, norm_w, 1e-5, H, G, D, V, batch, v_ref)
        got = kernels.delta_rule(u_ref, raw, small[:, 2:2 + H], log_decay, gate, norm_w, 1e-5, H, G, D, V, batch, v_got)
        _close(got, ref, 1e-4 if dtype == torch.float32 else 2e-2)
        _close(s_got, s_ref, 5e-5)
        if taps > 1:
            assert torch.equal(t_got, t_ref)
        assert torch.equal(s_got[[4, 7]], state[[4, 7]])
        kept_s, kept_t = s_got.clone(), t_got.clone()
        kernels.delta_rule(u_ref, raw, small[:, 2:2 + H], log_decay, gate, norm_w, 1e-5, H, G, D, V, batch, v_got, write_state=False)
        assert torch.equal(s_got, kept_s) and torch.equal(t_got, kept_t)
        state, tail = s_got, t_got


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,G,D,V", [(2, 1, 64, 64), (3, 3, 24, 40), (2, 2, 128, 32), (1, 1, 5, 7)])
def test_long_segments_run_as_parts(kernels, twin, dtype, H, G, D, V):
    """Segments of several hundred tokens are cut into parts that run side by side and are folded in order: the same
    outputs and end states as the walk token by token, beside short segments and single tokens, from states that are not zero."""
    g = torch.Generator().manual_seed(H * D + V)
    segs, slots = [(0, 300), (40, 1), (5, 700), (0, 64), (17, 257)], [3, 0, 4, 1, 2]
    batch = _batch(segs, slots)
    T = batch.num_tokens
    assert batch.max_seg_len >= kernels.MATRIX_STATE_PARTS_FROM
    # the delta rule
    C, taps = 2 * G * D + H * V, 3
    req = MatrixState(H, D, V, C, taps)
    state = (torch.randn(6, H, D, V, generator=g) * 0.5).to(DEV)
    tail = torch.randn(6, taps - 1, C, generator=g).to(DEV, dtype)
    u = torch.randn(T, C, generator=g).to(DEV, dtype)
    beta, gate = torch.randn(T, H, generator=g).to(DEV), torch.randn(T, H * V, generator=g).to(DEV)
    log_decay = -(torch.rand(T, H * D, generator=g) * 0.3).to(DEV)
    norm_w = (1 + 0.3 * torch.randn(V, generator=g)).to(DEV)
    s_ref, s_got, t_ref, t_got = state.clone(), state.clone(), tail.clone(), tail.clone()
    v_ref = req.view({"state": s_ref, "tail": t_ref}, slots=batch.seg_slot, slot_list=slots)
    v_got = req.view({"state": s_got, "tail": t_got}, slots=batch.seg_slot, slot_list=slots)
    ref = twin.delta_rule(u, u, beta, log_decay, gate, norm_w, 1e-5, H, G, D, V, batch, v_ref)
    got = kernels.delta_rule(u, u, beta, log_decay, gate, norm_w, 1e-5, H, G, D, V, batch, v_got)
    _close(got, ref, 2e-4 if dtype == torch.float32 else 2e-2)
    _close(s_got, s_ref, 2e-4)
    assert torch.equal(t_got, t_ref) and torch.equal(s_got[5], state[5])
    kept = s_got.clone()
    kernels.delta_rule(u, u, beta, log_decay, gate, norm_w, 1e-5, H, G, D, V, batch, v_got, write_state=False)
    assert torch.equal(s_got, kept) and torch.equal(t_got, t_ref)
    # the token-shift state
    width = 40
    req = MatrixState(H, D, D, width, 2)
    state = (torch.randn(6, H, D, D, generator=g) * 0.5).to(DEV)
    tail = torch.randn(6, 1, width, generator=g).to(DEV, dtype)
    rkvg = (torch.randn(T, 4, H * D, generator=g) * D ** -0.25).to(DEV, dtype)
    log_decay = -torch.exp(torch.randn(T, H * D, generator=g) * 1.5 - 2.5).to(DEV)
    bonus, norm_w = torch.randn(H, D, generator=g).to(DEV), (1 + 0.3 * torch.randn(H * D, generator=g)).to(DEV)
    x = torch.randn(T, width, generator=g).to(DEV, dtype)
    s_ref, s_got, t_ref, t_got = state.clone(), state.clone(), tail.clone(), tail.clone()
    v_ref = req.view({"state": s_ref, "tail": t_ref}, slots=batch.seg_slot, slot_list=slots)
    v_got = req.view({"state": s_got, "tail": t_got}, slots=batch.seg_slot, slot_list=slots)
    ref = twin.shifted_state(rkvg, log_decay, bonus, norm_w, 1e-5, H, D, x, batch, v_ref)
    got = kernels.shifted_state(rkvg, log_decay, bonus, norm_w, 1e-5, H, D, x, batch, v_got)
    _close(got, ref, 2e-4 if dtype == torch.float32 else 2e-2)
    _close(s_got, s_ref, 2e-4)
    assert torch.equal(t_got, t_ref) and torch.equal(s_got[5], state[5])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tokens_and_keys_made_to_stand_out(kernels, dtype):
    check_the_matrix_states_keep_a_far_token(kernels, DEV, dtype)
    check_the_bonus_is_for_the_current_token_only(kernels, DEV, dtype)
    check_one_latent_key_inside_the_window_only(kernels, DEV, dtype)
    check_a_far_row_of_the_distance_table(kernels, DEV, dtype)


# ---------------------------------------------------------------------------- attention with biases, a temperature and a distance table
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("heads,kv_heads,dim,vdim,page,far,rows", [
    (4, 2, 32, 16, 4, 40, 12), (1, 1, 10, 7, 8, 9, 5), (5, 5, 6, 9, 16, 3, 2), (6, 1, 16, 48, 16, 300, 8), (8, 2, 64, 64, 16, 100, 16),
    (4, 1, 128, 128, 16, 120, 16), (2, 2, 128, 128, 8, 20, 6), (6, 3, 64, 64, 32, 500, 32), (3, 1, 64, 128, 32, 64, 10)])
def test_biased_attention_against_its_twin(kernels, twin, dtype, heads, kv_heads, dim, vdim, page, far, rows):
    from tt_transformers_b200.parts.sink_attention import SinkAttention
    segs = [(0, 70), (129, 1), (63, 2), (64, 1), (0, 1), (300, 1), (127, 3), (page - 1, 2), (15, 40), (95, 3), (96, 1), (0, 2)]
    batch, view, qkv, g = _attention_setup(segs, heads, kv_heads, dim, vdim, page, None, None, dtype, seed=heads * dim + vdim)
    ref_view = PagedKV(kv_heads, dim, None, value_dim=vdim).view(
        {"keys": view.keys.clone(), "values": view.values.clone()}, block_table=view.block_table, page_size=page)
    ones = torch.ones(dim, device=DEV)
    bias = (torch.randn(qkv.shape[1], generator=g) * 0.5).to(DEV)
    rel = torch.randn(rows, heads, generator=g) * 1.5
    table = rel[torch.tensor([SinkAttention.distance_bucket(n, rows, far) for n in range(far + 1)])].t().contiguous().to(DEV)
    sinks = (torch.randn(heads, generator=g) * 2).to(DEV)
    for use_bias, temp in ((bias, (0.5, 64)), (None, (1.0, 1)), (bias, None)):
        a, b = qkv.clone(), qkv.clone()
        twin.qk_norm_rope_write(a, batch, ones, ones, 1e-5, None, 0, heads, kv_heads, dim, vdim, ref_view, bias=use_bias, q_temp=temp)
        kernels.qk_norm_rope_write(b, batch, ones, ones, 1e-5, None, 0, heads, kv_heads, dim, vdim, view, bias=use_bias, q_temp=temp)
        _close(b[:, :(heads + kv_heads) * dim], a[:, :(heads + kv_heads) * dim], TOL[dtype])
        written = ~torch.isnan(ref_view.keys.float())
        assert torch.equal(written, ~torch.isnan(view.keys.float()))
        _close(torch.where(written, view.keys.float(), 0), torch.where(written, ref_view.keys.float(), 0), TOL[dtype])
        wv = ~torch.isnan(ref_view.values.float())
        _close(torch.where(wv, view.values.float(), 0), torch.where(wv, ref_view.values.float(), 0), TOL[dtype])
        for cap, use_sinks, use_table in ((20.0, sinks, table), (None, sinks, table), (3.0, None, table), (None, sinks, None)):
            ref = twin.sink_attention(a, batch, heads, kv_heads, dim, vdim, 0.3, cap, use_sinks, ref_view, distance_bias=use_table)
            got = kernels.sink_attention(a, batch, heads, kv_heads, dim, vdim, 0.3, cap, use_sinks, ref_view, distance_bias=use_table)
            _close(got, ref, TOL[dtype])
    other = kernels.sink_attention(a, batch, heads, kv_heads, dim, vdim, 0.3, None, sinks, ref_view, distance_bias=table * 0.5)
    assert float((other.float() - ref.float()).abs().max()) > 0.02          # a table that is left out or halved shows


@pytest.mark.parametrize("heads,kv_heads,dim,page,far", [(8, 2, 64, 16, 120), (4, 1, 128, 16, 1000), (6, 3, 64, 32, 64)])
def test_biased_attention_over_long_contexts(kernels, twin, heads, kv_heads, dim, page, far):
    from tt_transformers_b200.parts.sink_attention import SinkAttention
    for segs in ([(1100, 1), (700, 1)], [(0, 700)], [(600, 3), (511, 2), (1023, 1), (1024, 1), (far - 1, 1), (far, 1), (far + 1, 2)]):
        batch, view, qkv, g = _attention_setup(segs, heads, kv_heads, dim, dim, page, None, None, torch.bfloat16, seed=dim + len(segs))
        rel = torch.randn(16, heads, generator=g) * 2
        table = rel[torch.tensor([SinkAttention.distance_bucket(n, 16, far) for n in range(far + 1)])].t().contiguous().to(DEV)
        sinks = (torch.randn(heads, generator=g) * 2 + 2).to(DEV)
        twin.qk_norm_rope_write(qkv, batch, None, None, 1e-5, None, 0, heads, kv_heads, dim, dim, view)
        ref = twin.sink_attention(qkv, batch, heads, kv_heads, dim, dim, 0.2, 25.0, sinks, view, distance_bias=table)
        _close(kernels.sink_attention(qkv, batch, heads, kv_heads, dim, dim, 0.2, 25.0, sinks, view, distance_bias=table), ref, 2e-2)


# ---------------------------------------------------------------------------- latent attention with a window and an amplitude
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("H,R,E,rot,page,window", [(4, 48, 16, 16, 4, 24), (1, 9, 6, 4, 8, 7), (5, 11, 0, 0, 16, 1), (4, 64, 32, 32, 16, 40),
                                                   (8, 128, 32, 32, 16, 96), (3, 9, 6, 4, 16, None), (16, 64, 64, 64, 16, 33)])
def test_latent_attention_with_a_window_against_its_twin(kernels, twin, dtype, H, R, E, rot, page, window):
    g = torch.Generator().manual_seed(H * R + E)
    segs = [(0, 70), (129, 1), (63, 2), (64, 1), (0, 1), (300, 1), (127, 3), (page - 1, 2), (15, 40), (95, 3), (96, 1)]
    width = max(-(-(p + n) // page) for p, n in segs)
    total = sum(-(-(p + n) // page) for p, n in segs)
    order = (torch.randperm(total, generator=g) + 1).tolist()
    rows = torch.full((total + 1, page, R + E), float("nan"))
    table = torch.zeros(len(segs), width, dtype=torch.int32)
    at = 0
    for r, (p, n) in enumerate(segs):
        for i in range(-(-(p + n) // page)):
            table[r, i] = order[at]
            fill = min(page, p - i * page)
            if fill > 0:
                rows[order[at], :fill] = torch.randn(fill, R + E, generator=g)
            at += 1
    batch = _batch(segs)
    T = batch.num_tokens
    inv_freq = (1.0 / 500.0 ** (torch.arange(0, rot, 2).float() / rot)).to(DEV) if rot else None
    norm_w = (1 + 0.3 * torch.randn(R, generator=g)).to(DEV)
    down = torch.randn(T, R + E + 3, generator=g).to(DEV)
    views = []
    for _ in range(2):
        views.append(LatentPages(R, E, window).view({"rows": rows.clone().to(DEV, dtype)}, block_table=table.to(DEV), page_size=page))
    for amplitude in (1.0, 1.139):
        assert twin.latent_prepare(down, batch, 0, R, E, None, norm_w, 1e-5, inv_freq, rot, views[0], True, dtype, amplitude=amplitude) is None
        assert kernels.latent_prepare(down, batch, 0, R, E, None, norm_w, 1e-5, inv_freq, rot, views[1], True, dtype, amplitude=amplitude) is None
        written = ~torch.isnan(views[0].rows.float())
        assert torch.equal(written, ~torch.isnan(views[1].rows.float()))
        _close(torch.where(written, views[1].rows.float(), 0), torch.where(written, views[0].rows.float(), 0), TOL[dtype])
        q_lat = (torch.randn(T, H, R, generator=g) * R ** -0.5).to(DEV, dtype)
        q_rot = torch.randn(T, H, E, generator=g).to(DEV, dtype) if E else None
        for use_window in (window, "view", (window or 10) + 5):
            ref = twin.latent_attention(q_lat, q_rot, batch, views[0], 0.4, None, inv_freq, rot, amplitude=amplitude, window=use_window)
            got = kernels.latent_attention(q_lat, q_rot, batch, views[0], 0.4, None, inv_freq, rot, amplitude=amplitude, window=use_window)
            _close(got, ref, TOL[dtype])
        w_uv = (torch.randn(H, 12, R, generator=g) * R ** -0.5).to(DEV, dtype)
        few = _batch(segs[1:7])
        lo = segs[0][1]
        few_view = LatentPages(R, E, window).view({"rows": views[0].rows}, block_table=views[0].block_table[1:7], page_size=page)
        n = few.num_tokens
        ref = twin.latent_attention_out(q_lat[lo:lo + n], q_rot[lo:lo + n] if E else None, few, few_view, 0.4, None, inv_freq, rot,
                                        w_uv, None, amplitude=amplitude, window=window)
        got = kernels.latent_attention_out(q_lat[lo:lo + n], q_rot[lo:lo + n] if E else None, few, few_view, 0.4, None, inv_freq, rot,
                                           w_uv, None, amplitude=amplitude, window=window)
        _close(got, ref, TOL[dtype])


# ---------------------------------------------------------------------------- the router with corrections and the experts
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("width,E,top,inter,shared,T", [(192, 10, 3, 80, 64, 70), (60, 1, 1, 20, None, 5), (128, 9, 1, 9, 5, 33),
                                                       (64, 8, 2, 48, 32, 300), (512, 32, 8, 128, 256, 1100), (48, 6, 6, 40, None, 3)])
def test_corrected_router_and_experts_against_their_twins(kernels, twin, dtype, width, E, top, inter, shared, T):
    g = torch.Generator().manual_seed(width + E)
    x = torch.randn(T, width, generator=g).to(DEV, dtype)
    w_r = (torch.randn(E, width, generator=g) * 4 * width ** -0.5).to(DEV)
    correction = (torch.randn(E, generator=g) * 0.3).to(DEV)
    c_ref, w_ref = twin.route_corrected(x, w_r, correction, E, top, 1.7, 1e-20)
    c_got, w_got = kernels.route_corrected(x, w_r, correction, E, top, 1.7, 1e-20)
    same = (c_got == c_ref).all(-1)
    assert float(same.float().mean()) > 0.99                    # a close call may go the other way in another order of summation
    _close(w_got[same], w_ref[same], 1e-5)
    assert float((w_got.sum(-1) - 1.7).abs().max()) < 1e-5
    plain_choice, _ = kernels.route_corrected(x, w_r, torch.zeros_like(correction), E, top, 1.7, 1e-20)
    if E > top and T > 30:
        assert not torch.equal(plain_choice, c_got)             # the corrections change choices
    w_gu = (torch.randn(E, 2 * inter, width, generator=g) * width ** -0.5).to(DEV, dtype)
    w_d = (torch.randn(E, width, inter, generator=g) * inter ** -0.5).to(DEV, dtype)
    sh = None
    if shared is not None:
        sh = ((torch.randn(2 * shared, width, generator=g) * width ** -0.5).to(DEV, dtype),
              (torch.randn(width, shared, generator=g) * shared ** -0.5).to(DEV, dtype), 0.0)
    rows = min(T, 48)            # the twin walks pair by pair
    ref = twin.routed_experts(x[:rows], c_got[:rows], w_got[:rows], w_gu, w_d, 0.0, 1.0, sh, None)
    got = kernels.routed_experts(x, c_got, w_got, w_gu, w_d, 0.0, 1.0, sh, None)
    _close(got[:rows], ref, TOL[dtype])
    few = kernels.routed_experts(x[:5], c_got[:5], w_got[:5], w_gu, w_d, 0.0, 1.0, sh, None)          # the matrix-vector form
    _close(few, ref[:5], TOL[dtype])


# ---------------------------------------------------------------------------- the whole engine
def _plain(cfg, w, toks):
    return plain_bufolorn.forward(cfg, w, toks).float()


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 6e-2)])
@pytest.mark.parametrize("name", ["ALIGNED", "ODD", "TENSOR"])
def test_engine_matches_the_plain_implementation(tmp_path, dtype, tol, name):
    folder = cases.write_folder(str(tmp_path / name), getattr(cases, name), seed=3,
                                dtype=torch.float32 if dtype == "float32" else torch.bfloat16)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 70 + i) for i, n in enumerate((37, 1, 19, 8, 26, 2, 140))}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        for graphs in (True, False):
            steps = make_steps(requests)
            pages = -(-helpers.max_live_tokens(requests, steps, rounding=16) // 16)
            engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=16, num_pages=pages, max_batch_size=4,
                                                       max_seq_len=256, cuda_graph=graphs, device=DEV))
            for grp in engine.cache.groups:
                if grp.pool is not None:
                    for t in grp.storage.values():
                        t.fill_(float("nan"))
            got = helpers.run_steps(engine, steps)
            engine.cache.audit()
            assert engine.cache.free_pages() == pages and engine.cache.free_slots == 4
            close = []
            for rid in ref:
                if dtype == "float32":
                    assert helpers.relative_error(got[rid], ref[rid]) < tol, (make_steps.__name__, graphs, rid)
                else:
                    # in bfloat16 a router's close call may go the other way for a token, and the states carry what that
                    # token wrote through the rest of its request: of all requests' rows nine in ten must agree, and the
                    # typical row closely
                    scale = float(ref[rid].abs().max())
                    close.append((got[rid] - ref[rid]).abs().amax(dim=-1) / scale)
            if close:
                rows = torch.cat(close)
                assert float((rows < tol).float().mean()) >= 0.9 and float(rows.median()) < tol / 2, (make_steps.__name__, graphs)
            engine.close()


@pytest.mark.parametrize("seed", [1, 4, 7, 10, 12, 15])
def test_configurations_drawn_from_a_seed(tmp_path, seed):
    """Sizes, head counts, layer order, windows, ranks, taps and constants that nobody chose by hand: whole prompts (one of
    300 tokens, which the walks cut into parts), mixed batches and decoded tails, in both precisions."""
    drawn = cases.random_config(seed)
    for dtype, tol in (("float32", 2e-4), ("bfloat16", 6e-2)):
        folder = cases.write_folder(str(tmp_path / dtype), drawn, seed=seed, dtype=torch.float32 if dtype == "float32" else torch.bfloat16)
        cfg, w = cases.read_folder(folder)
        requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, seed * 10 + i) for i, n in enumerate((33, 1, 300, 9, 70, 2))}
        ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
        for make_steps in (helpers.steps_whole, helpers.steps_mixed, helpers.steps_decode_tail):
            steps = make_steps(requests)
            pages = -(-helpers.max_live_tokens(requests, steps, rounding=16) // 16)
            engine = build_engine(folder, EngineConfig(dtype=dtype, page_size=16, num_pages=pages, max_batch_size=4, max_seq_len=512,
                                                       device=DEV))
            for grp in engine.cache.groups:
                if grp.pool is not None:
                    for t in grp.storage.values():
                        t.fill_(float("nan"))
            got = helpers.run_steps(engine, steps)
            engine.cache.audit()
            rows = torch.cat([(got[rid] - ref[rid]).abs().amax(dim=-1) / float(ref[rid].abs().max()) for rid in ref])
            if dtype == "float32":
                assert float(rows.max()) < tol, (make_steps.__name__, float(rows.max()))
            else:
                assert float((rows < tol).float().mean()) >= 0.9 and float(rows.median()) < tol / 2, make_steps.__name__
            engine.close()


def test_long_decoding_through_captured_steps(tmp_path):
    """300 decoded tokens after a prompt of 40, three requests side by side: states, convolution tails, kept inputs, window
    edges and the pages given back behind them, step after step through replays of captured steps."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=9)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], 340 - 7 * i, 20 + i) for i in range(3)}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    steps = helpers.steps_many(requests, live=3, tail=300, portion=(2, 40))
    engine = build_engine(folder, EngineConfig(dtype="float32", page_size=16, num_pages=3 * 22, max_batch_size=4, max_seq_len=512,
                                               device=DEV))
    got = helpers.run_steps(engine, steps)
    assert engine.graphs is not None and engine.graphs.replays >= 290
    places = helpers.wanted_positions(steps)
    for rid in ref:
        assert helpers.relative_error(got[rid], ref[rid][places[rid]]) < 2e-4, rid
    engine.cache.audit()


def test_greedy_generation_through_the_entry_point(tmp_path):
    from tt_transformers_b200.engine.llm import from_pretrained

    folder = cases.write_folder(str(tmp_path / "g"), cases.ODD, seed=7)
    cfg, w = cases.read_folder(folder)
    prompts = [helpers.random_tokens(cfg["vocab"], n, 80 + n) for n in (4, 13, 21, 50)]

    def plain_greedy(prompt, new):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(_plain(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p, 12) for p in prompts]
    # pages of 8 tokens, not enough for all four requests at their full length: one gives way and is recomputed
    llm = from_pretrained(folder, dtype="float32", page_size=8, num_pages=16, max_batch_size=4, max_seq_len=128,
                          max_step_tokens=32, max_chunk_tokens=16, device=DEV)
    assert llm.generate(prompts, max_new_tokens=12) == expect
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 16
