"""Bufolorn on the CPU: the configuration, the model as data, and the engine (step function, cache manager, scheduler)
with the plain twins of the kernels against the plain implementation of the design."""

import io
import json
import math
import os

import numpy as np
import pytest
import torch

import bufolorn_cases as cases
import helpers
import plain_bufolorn
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.config.base import ConfigError
from tt_transformers_b200.config.bufolorn import BufolornConfig, LatentConfig
from tt_transformers_b200.engine.step import StepEntry, build_engine
from tt_transformers_b200.models.bufolorn import model_spec
from tt_transformers_b200.parts.base import LatentPages, MatrixState, PagedKV
from tt_transformers_b200.parts.sink_attention import SinkAttention


def _plain(cfg, w, toks):
    return plain_bufolorn.forward(cfg, w, toks).float()


def _engine(folder, pages, page_size=4, slots=4, max_seq_len=128, **more):
    return build_engine(folder, EngineConfig(dtype="float32", page_size=page_size, num_pages=pages, max_batch_size=slots,
                                             max_seq_len=max_seq_len, device="cpu", **more), kernels=TorchKernels())


def _poison(engine):
    """What nobody has written reads as not-a-number: a key from a page that is not the request's shows."""
    for g in engine.cache.groups:
        if g.pool is not None:
            for t in g.storage.values():
                t.fill_(float("nan"))


# ---------------------------------------------------------------------------- configuration and model as data
def test_configuration_and_model_as_data():
    cfg = BufolornConfig.from_dict(cases.ALIGNED)
    assert cfg.residual_mult == 0.5 and cfg.embedding_scale == 3.0 and len(cfg.layers) == 5
    assert cfg.layers[3].mixer.kv_from == 1 and cfg.layers[3].mlp is None
    spec = model_spec(cfg)
    assert [c.cache_of for c in spec.order] == [None, None, None, 1, None]
    assert spec.layers[1].mixer.params["keep_window"] == 40          # the reader's window is the wider one
    assert spec.layers[0].mixer.kind == "mixer_pair" and spec.layers[0].mixer.params["combine"] == "weighted"
    assert spec.layers[3].block == "parallel_mixer_only" and spec.layers[2].feed_forward.kind == "corrected_experts"
    odd = model_spec(BufolornConfig.from_dict(cases.ODD))
    assert odd.layers[1].mixer.params["keep_window"] is None        # a reader that sees everything keeps everything
    assert odd.layers[3].position is None                           # no rotated part, no encoding
    bare = BufolornConfig.from_dict(cases.without_sizes_of_made_up_tensors(cases.ALIGNED))
    assert bare.layers[2].mixer.decay_rank is None and bare.layers[0].mixer.left.bias_rows is None


@pytest.mark.parametrize("breaker,match", [
    (lambda c: c["layers"][0].update(type="conv"), "type 'conv' is not known"),
    (lambda c: c["layers"][0]["mixer"]["left"].pop("bias_max"), "bias_max"),
    (lambda c: c["layers"][0]["mixer"]["left"].update(heads=3), "multiple of 'kv_heads'"),
    (lambda c: c["layers"][3]["mixer"].update(kv_from=3), "must name an earlier layer"),
    (lambda c: c["layers"][3]["mixer"].update(kv_from=0), "latent_attention layer"),
    (lambda c: c["layers"][3]["mixer"].update(kv_rank=40), "must equal those of layer 1"),
    (lambda c: c["layers"][1]["mixer"]["rot"].update(dims=18), "rot.dims"),
    (lambda c: c["layers"][1]["mlp"]["router"].update(top=9), "'top' must lie between"),
    (lambda c: c["layers"][2]["mixer"].pop("conv"), "'conv' is missing"),
    (lambda c: c.pop("norm"), "'norm' must be an object"),
])
def test_configuration_errors_name_the_key(breaker, match):
    import copy
    cfg = copy.deepcopy(cases.ALIGNED)
    breaker(cfg)
    with pytest.raises(ConfigError, match=match):
        BufolornConfig.from_dict(cfg)


def test_distance_buckets():
    """Single positions below half the rows, logarithmic steps up to `far`, the last row from there on."""
    rows, far = 12, 40
    got = [SinkAttention.distance_bucket(n, rows, far) for n in range(60)]
    assert got[:6] == list(range(6)) and got[6] == 6 and got[39] <= 11 and got[40:] == [11] * 20
    assert all(b >= a for a, b in zip(got, got[1:]))
    for n in range(6, 40):
        assert got[n] == 6 + int(math.floor(math.log(n / 6) / math.log(40 / 6) * 6))
    assert [SinkAttention.distance_bucket(n, 5, 9) for n in (0, 1, 2, 3, 8, 9, 100)] == [0, 1, 2, 2, 4, 4, 4]


# ---------------------------------------------------------------------------- each mechanism alone, and whole models
@pytest.mark.parametrize("kind", ["delta", "side_by_side", "latent", "shared_latent", "dense", "moe"])
def test_each_mechanism_alone(tmp_path, kind):
    folder = cases.write_folder(str(tmp_path / kind), cases.single(kind), seed=11)
    cfg, w = cases.read_folder(folder)
    requests = {"a": helpers.random_tokens(cfg["vocab"], 41, 5), "b": helpers.random_tokens(cfg["vocab"], 3, 6)}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_portions, helpers.steps_mixed):
        engine = _engine(folder, pages=16)
        _poison(engine)
        got = helpers.run_steps(engine, make_steps(requests))
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 2e-5, (kind, make_steps.__name__, rid)


@pytest.mark.parametrize("name", ["ALIGNED", "ODD"])
def test_engine_with_plain_twins_matches_the_plain_implementation(tmp_path, name):
    """Whole prompts, decoded tails, portions down to two tokens and mixed batches on a pool that holds just what is live:
    pages and slots are freed and used again."""
    folder = cases.write_folder(str(tmp_path / name), getattr(cases, name), seed=3)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 70 + i) for i, n in enumerate((37, 1, 19, 8, 26, 2, 90))}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        steps = make_steps(requests)
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=4) // 4)
        engine = _engine(folder, pages=pages)
        _poison(engine)
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        assert engine.cache.free_pages() == pages and engine.cache.free_slots == 4
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 3e-5, (make_steps.__name__, rid)


@pytest.mark.parametrize("seed", [2, 5, 11])
def test_configurations_drawn_from_a_seed(tmp_path, seed):
    """Sizes, head counts, layer order, windows, ranks, taps and constants that nobody chose by hand."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.random_config(seed), seed=seed)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, seed * 10 + i) for i, n in enumerate((33, 1, 70, 9, 2))}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_mixed):
        steps = make_steps(requests)
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=4) // 4)
        engine = _engine(folder, pages=pages)
        _poison(engine)
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 5e-5, (make_steps.__name__, rid)


def test_token_by_token_from_the_first_token_and_a_long_decoded_tail(tmp_path):
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=5)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 120, 1)
    ref = _plain(cfg, w, toks)
    engine = _engine(folder, pages=30)
    _poison(engine)
    rows = [engine.step([StepEntry("a", [t], [0])])[0] for t in toks]
    assert helpers.relative_error(torch.stack(rows), ref) < 3e-5


def test_pages_behind_the_widest_window_are_given_back(tmp_path):
    """The latent cache keeps the reader's window of 40, not the owner's 24; the attention beside the state keeps everything."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=5)
    engine = _engine(folder, pages=40, max_seq_len=160)
    engine.step([StepEntry("a", helpers.random_tokens(300, 150, 2), [149])])
    by_request = {type(g.request): g for g in engine.cache.groups}
    assert by_request[LatentPages].request.window == 40
    assert by_request[LatentPages].pool.held_count == -(-150 // 4) - (150 - 1 - 40 + 1) // 4
    assert by_request[PagedKV].pool.held_count == -(-150 // 4)
    assert isinstance(by_request[MatrixState].request, MatrixState)
    engine.finish("a")
    engine.cache.audit()
    assert engine.cache.free_pages() == 40 and engine.cache.free_slots == 4


# ---------------------------------------------------------------------------- mechanisms with inputs made to show a fault
def _batch(segs, device, slots=None):
    """segs: [(cached tokens, new tokens)] -> what the kernels read of a StepBatch."""
    from types import SimpleNamespace

    lens, pos0 = [n for _, n in segs], [p for p, _ in segs]
    slots = slots if slots is not None else list(range(len(segs)))
    cu = [0]
    for n in lens:
        cu.append(cu[-1] + n)
    i32 = dict(dtype=torch.int32, device=device)
    return SimpleNamespace(
        positions=torch.cat([torch.arange(p, p + n) for p, n in segs]).to(**i32),
        seg_of_token=torch.cat([torch.full((n,), r) for r, n in enumerate(lens)]).to(**i32),
        cu_seqlens=torch.tensor(cu, **i32), seg_pos0=torch.tensor(pos0, **i32), seg_slot=torch.tensor(slots, **i32),
        seg_lens=lens, seg_pos0_list=pos0, seg_slot_list=slots, num_segments=len(segs), num_tokens=cu[-1],
        max_seg_len=max(lens), max_context=max(p + n for p, n in segs), extras={})


def _latent_setup(device, dtype, R, E, page, pos0, new):
    """A latent cache of one request with pos0 cached rows, all zero but what a test puts there."""
    ctx = pos0 + new
    n_pages = -(-ctx // page)
    order = (torch.randperm(n_pages, generator=torch.Generator().manual_seed(ctx)) + 1)
    rows = torch.zeros(n_pages + 1, page, R + E, device=device, dtype=dtype)
    table = order.to(torch.int32).view(1, n_pages).to(device)
    view = LatentPages(R, E, None).view({"rows": rows}, block_table=table, page_size=page)

    def put(pos, vector):
        rows[int(order[pos // page]), pos % page] = vector.to(device, dtype)
    return view, put


def check_one_latent_key_inside_the_window_only(kernels, device, dtype=torch.float32):
    """One cached row stands out (its score beats all others by far); a query sees it exactly while it lies inside the
    window: at distance window - 1 the output is that row's latent, at distance window it is not, in prompts and decoding."""
    R, E, H, page, window = 16, 0, 2, 8, 11
    key_at = 20
    special = torch.zeros(R)
    special[0], special[1] = 8.0, 3.0
    for pos0, new in ((key_at + window - 1, 1), (key_at + window, 1), (key_at + 1, window + 3), (key_at + window - 3, 4)):
        view, put = _latent_setup(device, dtype, R, E, page, pos0, new)
        for p in range(pos0 + new):
            filler = torch.zeros(R)
            filler[2] = 1.0
            put(p, filler)
        put(key_at, special)
        batch = _batch([(pos0, new)], device)
        q = torch.zeros(new, H, R, device=device, dtype=dtype)
        q[:, :, 0] = 4.0                                     # score 32 for the special row, 0 for the others
        out = kernels.latent_attention(q, None, batch, view, 1.0, None, None, 0, window=window).float().cpu()
        for i in range(new):
            inside = pos0 + i - key_at < window
            assert abs(float(out[i, 0, 1]) - (3.0 if inside else 0.0)) < 0.05, (pos0, new, i)
            assert abs(float(out[i, 0, 2]) - (0.0 if inside else 1.0)) < 0.05, (pos0, new, i)


def test_one_latent_key_inside_the_window_only():
    check_one_latent_key_inside_the_window_only(TorchKernels(), "cpu")


def check_a_far_row_of_the_distance_table(kernels, device, dtype=torch.float32):
    """Among several hundred keys with equal scores the last row of the distance table lifts every key from the first
    distance that reaches that row (before `far`) on: the output is the mean of their values; a sink as large takes half of
    the weight; a sink left out would show."""
    heads, kv_heads, dim, vdim, page, far, rows = 2, 1, 8, 4, 16, 37, 10
    ctx = 400
    g = torch.Generator().manual_seed(1)
    n_pages = -(-ctx // page)
    table = (torch.randperm(n_pages, generator=g) + 1).to(torch.int32).view(1, n_pages).to(device)
    view = PagedKV(kv_heads, dim, None, value_dim=vdim).view(
        {"keys": torch.zeros(n_pages + 1, kv_heads, page, dim, device=device, dtype=dtype),       # every score is zero before the bias
         "values": torch.zeros(n_pages + 1, kv_heads, page, vdim, device=device, dtype=dtype)}, block_table=table, page_size=page)
    batch = _batch([(ctx - 1, 1)], device)
    qkv = torch.zeros(1, (heads + kv_heads) * dim + kv_heads * vdim, device=device, dtype=dtype)
    values = torch.randn(ctx, vdim, generator=g)
    for p in range(ctx):
        view.values[int(view.block_table[0, p // page]), 0, p % page] = values[p].to(device, dtype)
    qkv[:, (heads + kv_heads) * dim:] = values[ctx - 1].to(device, dtype)
    rel = torch.zeros(rows, heads)
    rel[rows - 1, 0] = 30.0                                      # head 0: everything at `far` or beyond; head 1: no bias at all
    buckets = [SinkAttention.distance_bucket(n, rows, far) for n in range(far + 1)]
    table = rel[torch.tensor(buckets)].t().contiguous().to(device)
    far = buckets.index(rows - 1)                                # the first distance in the last row
    assert far < 37
    kernels.qk_norm_rope_write(qkv, batch, None, None, 1e-5, None, 0, heads, kv_heads, dim, vdim, view)
    out = kernels.sink_attention(qkv, batch, heads, kv_heads, dim, vdim, 1.0, None, None, view, distance_bias=table).float().cpu()
    stored = torch.stack([view.values[int(view.block_table[0, p // page]), 0, p % page].float().cpu() for p in range(ctx)])
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert float((out[0, :vdim] - stored[:ctx - far].mean(0)).abs().max()) < tol
    assert float((out[0, vdim:] - stored.mean(0)).abs().max()) < tol
    sinks = torch.tensor([30.0 + math.log(ctx - far), -30.0]).to(device)
    half = kernels.sink_attention(qkv, batch, heads, kv_heads, dim, vdim, 1.0, None, sinks, view, distance_bias=table).float().cpu()
    assert float((half[0, :vdim] - 0.5 * stored[:ctx - far].mean(0)).abs().max()) < tol
    assert float((half[0, vdim:] - stored.mean(0)).abs().max()) < tol


def test_a_far_row_of_the_distance_table():
    check_a_far_row_of_the_distance_table(TorchKernels(), "cpu")


def check_the_matrix_states_keep_a_far_token(kernels, device, dtype=torch.float32):
    """A value written at a request's first token under its own key comes back hundreds of tokens later, through steps of
    any size, when nothing decays and no other token writes under that key; the delta rule replaces it when the key is
    written again, and forgets it when the key's channel decays."""
    H, G, D, V, taps = 2, 1, 4, 3, 1
    C = 2 * G * D + H * V
    req = MatrixState(H, D, V, C, taps)
    value = torch.tensor([1.0, -2.0, 3.0])

    def run(decay_first_channel, write_again):
        state = torch.zeros(3, H, D, V, device=device)
        tail = torch.zeros(3, 1, C, device=device, dtype=dtype)
        outs, pos = [], 0
        for new in (1, 7, 200, 1, 1, 64, 2, 1):
            batch = _batch([(pos, new)], device, slots=[1])
            view = req.view({"state": state, "tail": tail}, slots=batch.seg_slot, slot_list=[1])
            u = torch.zeros(new, C, device=device, dtype=dtype)
            u[:, 0] = 2.0                                   # every query asks for key channel 0
            u[:, D + 1] = 5.0                               # every later token writes under key channel 1 ...
            u[:, 2 * D:] = 9.0                              # ... some other value
            beta = torch.full((new, H), 30.0, device=device)
            if pos == 0:
                u[0, D + 1], u[0, D] = 0.0, 3.0             # the first token writes `value` under key channel 0
                u[0, 2 * D:2 * D + V] = value.to(device, dtype)
                u[0, 2 * D + V:] = value.to(device, dtype)
            if write_again and pos + new == 276:            # the last token but one of the 64 writes under channel 0 again
                u[-1, D + 1], u[-1, D] = 0.0, 1.0
                u[-1, 2 * D:] = -value.repeat(H).to(device, dtype)
            log_decay = torch.zeros(new, H * D, device=device)
            if decay_first_channel:
                log_decay[:, 0] = -0.1                      # head 0 forgets channel 0; head 1 keeps it
            gate = torch.full((new, H * V), 30.0, device=device)
            outs.append(kernels.delta_rule(u, u, beta, log_decay, gate, torch.ones(V, device=device), 1e-6, H, G, D, V, batch,
                                           view).float().cpu())
            pos += new
        return torch.cat(outs).view(-1, H, V)

    unit = value / torch.sqrt((value * value).mean())       # the head norm leaves the direction
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    kept = run(False, False)
    for t in (0, 1, 8, 207, 276):
        assert float((kept[t] - unit).abs().max()) < tol, t
    again = run(False, True)
    assert float((again[274, 0] - unit).abs().max()) < tol and float((again[276, 0] + unit).abs().max()) < tol
    gone = run(True, False)
    assert float((gone[276, 1] - unit).abs().max()) < tol                     # head 1 keeps it
    assert float(gone[276, 0].abs().max()) < 1e-6 and float((gone[5, 0] - unit).abs().max()) < tol  # head 0 has forgotten it by then


def test_the_matrix_states_keep_a_far_token():
    check_the_matrix_states_keep_a_far_token(TorchKernels(), "cpu")


def check_the_bonus_is_for_the_current_token_only(kernels, device, dtype=torch.float32):
    """From an empty state the first output is (sum_d r_d u_d k_d) v; the second token reads the first without the bonus."""
    H, D, width = 1, 4, 6
    req = MatrixState(H, D, D, width, 2)
    state = torch.zeros(2, H, D, D, device=device)
    tail = torch.zeros(2, 1, width, device=device, dtype=dtype)
    batch = _batch([(0, 2)], device, slots=[0])
    view = req.view({"state": state, "tail": tail}, slots=batch.seg_slot, slot_list=[0])
    rkvg = torch.zeros(2, 4, H * D, device=device, dtype=dtype)
    rkvg[:, 0, 0] = 1.0                                     # r = e0
    rkvg[0, 1, 0] = 2.0                                     # the first token's key e0 * 2, value below; the second writes nothing
    rkvg[0, 2] = torch.tensor([1.0, 2.0, -1.0, 0.5]).to(device, dtype)
    rkvg[:, 3] = 30.0                                       # silu(30) = 30
    bonus = torch.tensor([[0.25, 9.0, 9.0, 9.0]], device=device)
    x = torch.randn(2, width).to(device, dtype)
    raw = kernels.shifted_state(rkvg, torch.zeros(2, H * D, device=device), bonus, torch.ones(H * D, device=device), 0.0, H, D,
                                x, batch, view).float().cpu()
    v = torch.tensor([1.0, 2.0, -1.0, 0.5])
    unit = v / torch.sqrt((v * v).mean()) * 30.0
    assert float((raw[0] - unit).abs().max()) < 0.2 and float((raw[1] - unit).abs().max()) < 0.2     # the same direction twice ...
    assert float((state[0, 0, 0].cpu() - 2.0 * v).abs().max()) < 1e-2                                    # ... and k v^T in the state, without the bonus
    assert float((tail[0, 0].float().cpu() - x[1].float().cpu()).abs().max()) == 0.0                     # the last input is kept


def test_the_bonus_is_for_the_current_token_only():
    check_the_bonus_is_for_the_current_token_only(TorchKernels(), "cpu")


def test_corrections_steer_the_choice_and_not_the_weights():
    k = TorchKernels()
    x = torch.tensor([[1.0, 0.0], [0.0, 1.0]])
    w_r = torch.tensor([[2.0, -2.0], [1.0, 1.0], [0.0, 3.0]])
    s = torch.sigmoid(x @ w_r.t())
    choice, weight = k.route_corrected(x, w_r, torch.tensor([0.0, 0.0, 0.0]), 3, 2, 1.5, 1e-20)
    assert choice.tolist() == [[0, 1], [2, 1]]
    choice, weight = k.route_corrected(x, w_r, torch.tensor([-1.0, 0.0, 0.6]), 3, 2, 1.5, 1e-20)
    assert choice.tolist() == [[2, 1], [2, 1]]
    assert torch.allclose(weight[0], torch.stack([s[0, 2], s[0, 1]]) / (s[0, 2] + s[0, 1]) * 1.5)


# ---------------------------------------------------------------------------- the runner and the entry point
def test_trace_replay_of_a_bufolorn_folder(tmp_path):
    from tt_transformers_b200.engine.trace import run_trace

    folder = cases.write_folder(str(tmp_path / "m"), cases.ODD, seed=2)
    cfg, w = cases.read_folder(folder)
    requests = {"a": helpers.random_tokens(cfg["vocab"], 30, 1), "b": helpers.random_tokens(cfg["vocab"], 9, 2)}
    steps = helpers.steps_mixed(requests, decode_tail=4)
    lines = [json.dumps({"step": i, "entries": s["entries"], "end": s["end"]}) for i, s in enumerate(steps)]
    out, log = str(tmp_path / "out"), io.StringIO()
    run_trace(folder, "float32", out, 128, lines, log=log, device="cpu", kernels=TorchKernels(), cuda_graph=False)
    assert log.getvalue().split() == [x for i in range(len(steps)) for x in ("done", str(i))]
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    at = {rid: 0 for rid in requests}
    for i, s in enumerate(steps):
        rows = np.fromfile(os.path.join(out, f"{i}.f32"), dtype="<f4").reshape(-1, cfg["vocab"])
        row = 0
        for e in s["entries"]:
            for wpos in e["want"]:
                expect = ref[e["id"]][at[e["id"]] + wpos]
                assert float((torch.from_numpy(rows[row].copy()) - expect).abs().max()) / float(expect.abs().max()) < 3e-5
                row += 1
            at[e["id"]] += len(e["tokens"])


def test_greedy_generation_through_the_scheduler_under_page_pressure(tmp_path):
    from tt_transformers_b200.engine.llm import from_pretrained

    folder = cases.write_folder(str(tmp_path / "g"), cases.single("shared_latent"), seed=7)
    cfg, w = cases.read_folder(folder)
    prompts = [helpers.random_tokens(cfg["vocab"], n, 80 + n) for n in (4, 13, 21)]

    def plain_greedy(prompt, new):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(_plain(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p, 8) for p in prompts]
    # 7 pages of 8 tokens for requests that end at 12, 21 and 29 tokens: they cannot all stay, one gives way and is recomputed
    llm = from_pretrained(folder, dtype="float32", page_size=8, num_pages=7, max_batch_size=3, max_seq_len=64,
                          max_step_tokens=16, max_chunk_tokens=8, device="cpu", kernels=TorchKernels())
    assert llm.generate(prompts, max_new_tokens=8) == expect
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 7
