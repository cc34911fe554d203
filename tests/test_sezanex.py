"""Sezanex on the CPU: configuration, model as data, and the engine's step function, cache manager, scheduler and
trace replay with the kernels' plain twins against the plain implementation."""

import io
import json
import math

import numpy as np
import pytest
import torch

import helpers
import plain_sezanex
import sezanex_cases as cases
from torch_kernels import TorchKernels
from tt_transformers_b200.config import EngineConfig
from tt_transformers_b200.config.base import ConfigError
from tt_transformers_b200.engine.step import StepEntry, build_engine
from tt_transformers_b200.engine.trace import run_trace
from tt_transformers_b200.parts import DecoderModel, PagedKV
from tt_transformers_b200.parts.base import MatrixState
from tt_transformers_b200.registry import architecture_of, get_architecture


def _plain(cfg, w, toks):
    return plain_sezanex.forward(cfg, w, toks).float()


def _engine(folder, pages, page_size=4, slots=4, max_seq_len=128, **more):
    return build_engine(folder, EngineConfig(dtype="float32", page_size=page_size, num_pages=pages, max_batch_size=slots,
                                             max_seq_len=max_seq_len, device="cpu", **more), kernels=TorchKernels())


def _poison(engine):
    """What a page or a slot held before must never be read: NaN everywhere (admission zeroes a slot's state)."""
    for g in engine.cache.groups:
        for t in g.storage.values():
            t.fill_(float("nan"))


def test_configuration_and_model_as_data():
    arch = get_architecture(architecture_of(cases.ALIGNED))
    cfg = arch.load_config(cases.ALIGNED)
    assert [l.type for l in cfg.layers] == ["attention", "mamba2", "attention", "mamba2"]
    assert (cfg.loop_start, cfg.loop_stop, cfg.loop_times) == (1, 3, 3)
    assert cfg.layers[2].mixer.kv_heads == 1 and cfg.layers[2].mixer.window == 9 and cfg.layers[2].mlp is None
    assert cfg.layers[2].mixer.yarn.slow == 0.5 and cfg.layers[0].mixer.yarn.original == 64
    assert cfg.layers[1].mixer.taps == 4 and cfg.layers[3].mixer.norm_groups == 4
    assert cfg.layers[1].mlp.top == 2 and cfg.layers[0].mlp.kind == "dense" and cfg.layers[0].mlp.inter == 160
    spec = arch.model_spec(cfg)
    assert [c.layer for c in spec.order] == [0, 1, 2, 1, 2, 1, 2, 3]
    assert [at for at, _ in spec.stream_steps] == [1, 3, 5]                       # a matrix before every pass, the first too
    assert all(s.kind == "pass_mix" for _, s in spec.stream_steps)
    model = DecoderModel(spec)
    requests = model.cache_requests()
    assert requests[0] == PagedKV(2, 32, 24, value_dim=16)
    assert requests[1] == requests[3] == requests[5] == MatrixState(4, 24, 16, 4 * 16 + 2 * 2 * 24, 4)  # a state per pass
    assert requests[2] == requests[4] == PagedKV(1, 16, 9, value_dim=48)
    assert requests[7] == MatrixState(2, 8, 48, 2 * 48 + 2 * 8, 3)
    names = {s.name: s.shape for s in model.tensor_specs()}
    assert names["loop.in"] == (128, 256) and names["l0.norm1.alpha"] == () and names["l0.norm2b.b"] == (128,)
    assert names["l0.mix.q.norm"] == (128,) and names["l0.mix.k.norm"] == (64,) and names["l0.mix.v"] == (32, 128)
    assert names["l2.mix.o"] == (128, 288) and names["l1.mix.in"] == (2 * 64 + 2 * 48 + 4, 128)
    assert names["l1.mix.conv"] == (64 + 96, 4) and names["l1.mix.conv.b"] == (160,) and names["l3.mix.norm"] == (96,)
    assert names["l1.mix.A_log"] == names["l1.mix.D"] == names["l1.mix.dt_bias"] == (4,)
    assert names["l1.mlp.e7.gate"] == (48, 128) and names["l3.mlp.router"] == (6, 128) and names["l0.mlp.up"] == (160, 128)
    assert "l2.mlp.router" not in names and "l2.norm2" not in names and "head" not in names and "final.norm.alpha" in names
    # a model without a loop has neither passes nor their matrix; a layer without a rotation has no position part
    plain_spec = arch.model_spec(arch.load_config(cases.PLAIN))
    assert plain_spec.stream_steps == () and "loop.in" not in {s.name for s in DecoderModel(plain_spec).tensor_specs()}
    assert plain_spec.layers[2].position is None and plain_spec.layers[0].position.params["scaling"] is None
    assert DecoderModel(plain_spec).cache_requests()[2] == PagedKV(2, 8, None, value_dim=8)
    # cut short, the model keeps the passes that still start
    assert [at for at, _ in spec.first_entries(4).stream_steps] == [1, 3]


@pytest.mark.parametrize("breaker,match", [
    (lambda c: c["layers"][0].update(type="ring"), "not known"),
    (lambda c: c["layers"][1]["mixer"].pop("state"), "state"),
    (lambda c: c["layers"][1]["mixer"].update(groups=3), "groups"),
    (lambda c: c["layers"][3]["mixer"].update(norm_groups=5), "norm_groups"),
    (lambda c: c["layers"][0]["mixer"]["rot"].update(dims=7), "rot.dims"),
    (lambda c: c["layers"][0]["mixer"]["rot"]["scaling"].pop("fast"), "fast"),
    (lambda c: c["layers"][0]["mixer"].update(kv_heads=3), "kv_heads"),
    (lambda c: c["layers"][0]["mixer"].pop("scale"), "scale"),
    (lambda c: c["layers"][1]["mlp"]["router"].update(top=9), "top"),
    (lambda c: c["layers"][0]["mlp"].update(kind="glu"), "not known"),
    (lambda c: c["loop"].update(stop=9), "loop"),
    (lambda c: c.pop("norm"), "norm"),
])
def test_configuration_errors_name_the_key(breaker, match):
    cfg = json.loads(json.dumps(cases.ALIGNED))
    breaker(cfg)
    with pytest.raises(ConfigError, match=match):
        get_architecture("Sezanex").load_config(cfg)


@pytest.mark.parametrize("kind", ["attention", "mamba2", "dense", "moe"])
def test_each_mechanism_alone(tmp_path, kind):
    folder = cases.write_folder(str(tmp_path / kind), cases.single(kind), seed=11)
    cfg, w = cases.read_folder(folder)
    requests = {"a": helpers.random_tokens(cfg["vocab"], 33, 1), "b": helpers.random_tokens(cfg["vocab"], 12, 2)}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_portions, helpers.steps_decode_tail):
        engine = _engine(folder, pages=12)
        _poison(engine)
        got = helpers.run_steps(engine, make_steps(requests))
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 2e-5, (make_steps.__name__, rid)


@pytest.mark.parametrize("name", ["ALIGNED", "ODD", "PLAIN"])
def test_engine_with_plain_twins_matches_the_plain_implementation(tmp_path, name):
    """Whole prompts, prompts with decoded tails, portions down to two tokens, and mixed batches of unequal requests
    on a pool that holds just what is live, with six requests on four slots: pages and slots are used again."""
    folder = cases.write_folder(str(tmp_path / name), getattr(cases, name), seed=3)
    cfg, w = cases.read_folder(folder)
    requests = {f"r{i}": helpers.random_tokens(cfg["vocab"], n, 70 + i) for i, n in enumerate((37, 1, 19, 8, 26, 2))}
    ref = {rid: _plain(cfg, w, toks) for rid, toks in requests.items()}
    for make_steps in (helpers.steps_whole, helpers.steps_decode_tail, helpers.steps_portions, helpers.steps_mixed):
        steps = make_steps(requests)
        pages = -(-helpers.max_live_tokens(requests, steps, rounding=4) // 4)
        engine = _engine(folder, pages=pages, max_seq_len=64)
        _poison(engine)
        got = helpers.run_steps(engine, steps)
        engine.cache.audit()
        assert engine.cache.free_pages() == pages and engine.cache.free_slots == 4
        for rid in ref:
            assert helpers.relative_error(got[rid], ref[rid]) < 2e-5, (make_steps.__name__, rid)


def test_token_by_token_from_the_first_token_and_a_long_decoded_tail(tmp_path):
    """Every token alone from position 0 on (the state starts at zero, the convolution sees zeros before the start, the
    first keys stand alone beside the constant in the denominator), 150 decoded tokens behind a short prompt (windows
    of 24 and 9 positions pass over decoded tokens many times, the state-space layers carry 150 updates)."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=8)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 156, 5)
    ref = _plain(cfg, w, toks)
    for first in (1, 6):
        engine = _engine(folder, pages=14, max_seq_len=256)      # 156 tokens would need 39 pages without giving back
        _poison(engine)
        rows = [engine.step([StepEntry("a", toks[:first], list(range(first)))])]
        for t in toks[first:]:
            rows.append(engine.step([StepEntry("a", [t], [0])]))
        assert helpers.relative_error(torch.cat(rows), ref) < 3e-5, first
        engine.finish("a")
        engine.cache.audit()
        assert engine.cache.free_pages() == 14


def test_pages_behind_the_window_are_given_back(tmp_path):
    """Windows of 24 positions (layer 0) and of 9 (layer 2) on pages of 4: a request of 70 tokens never holds more
    pages per group than its window needs, plus the portion that is being written."""
    folder = cases.write_folder(str(tmp_path / "m"), cases.ALIGNED, seed=5)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 70, 4)
    ref = _plain(cfg, w, toks)
    engine = _engine(folder, pages=16, max_seq_len=128)
    _poison(engine)
    rows, at = [], 0
    for n in [5, 2, 9, 1, 1, 17, 3, 1, 1, 1, 2, 20, 1, 1, 5]:
        rows.append(engine.step([StepEntry("a", toks[at:at + n], list(range(n)))]))
        at += n
    assert at == 70
    assert engine.cache.free_pages() >= 16 - 8                   # 24 positions behind the end on pages of 4, and its edges
    assert helpers.relative_error(torch.cat(rows), ref) < 2e-5
    engine.finish("a")
    engine.cache.audit()
    assert engine.cache.free_pages() == 16


def _window_setup(device, window, page, pos0, new, kv_heads, dim, vdim):
    """One request with pos0 cached tokens and `new` new ones on pages in descending order (the table is used)."""
    from types import SimpleNamespace

    ctx = pos0 + new
    n_pages = -(-ctx // page)
    order = list(range(n_pages, 0, -1))
    keys = torch.full((n_pages + 1, kv_heads, page, dim), float("nan"), device=device)
    values = torch.full((n_pages + 1, kv_heads, page, vdim), float("nan"), device=device)
    table = torch.tensor([order], dtype=torch.int32, device=device)
    view = PagedKV(kv_heads, dim, window, value_dim=vdim).view({"keys": keys, "values": values}, block_table=table, page_size=page)

    def batch(p0, n):
        return SimpleNamespace(positions=torch.arange(p0, p0 + n, dtype=torch.int32, device=device),
                               seg_of_token=torch.zeros(n, dtype=torch.int32, device=device), seg_lens=[n], seg_pos0_list=[p0],
                               cu_seqlens=torch.tensor([0, n], dtype=torch.int32, device=device), num_segments=1,
                               seg_pos0=torch.tensor([p0], dtype=torch.int32, device=device), num_tokens=n, max_seg_len=n,
                               max_context=p0 + n, extras={})
    return view, batch


def check_one_key_inside_the_window_only(kernels, device, dtype=torch.float32, sizes=(2, 1, 8, 4, 4, 11), cases_=None):
    """A query whose score with one key stands out returns that key's value if the key is one of the last `window`
    positions (the oldest of them, a page's first and last row, the query's own position), and nothing of it if it
    lies one position further back: then the window's keys all score zero beside the constant one in the denominator,
    so the output is the sum of their values over (their number + 1). For a decoded token, for the last token of a
    portion, and for the first tokens of a sequence, where fewer keys than the window exist."""
    heads, kv_heads, dim, vdim, page, window = sizes
    sinks = torch.zeros(heads, device=device)
    tol = 2e-2 if dtype != torch.float32 else 1e-5
    for pos0, new in cases_ or ((40, 1), (38, 3), (36, 1), (35, 2), (0, 30), (0, 1), (0, 3), (9, 2), (10, 1), (11, 1)):
        last = pos0 + new - 1
        start = max(0, last - window + 1)                        # the oldest position that `last` sees
        for far in sorted({start, start - 1, start + 1, last, max(start, last - 1), (start // page + 1) * page,
                           (start // page + 1) * page - 1, 0}):
            if far < 0 or far > last:
                continue
            view, batch = _window_setup(device, window, page, pos0, new, kv_heads, dim, vdim)
            view.keys, view.values = view.keys.to(dtype), view.values.to(dtype)
            ctx = pos0 + new
            g = torch.Generator().manual_seed(far)
            k_all = torch.zeros(ctx, kv_heads * dim)
            for kv in range(kv_heads):
                k_all[far, kv * dim] = 6.0
            v_all = torch.randn(ctx, kv_heads * vdim, generator=g)
            q = torch.zeros(ctx, heads * dim)
            for h in range(heads):
                q[:, h * dim] = 6.0
            qkv = torch.cat([q, k_all, v_all], 1).to(device, dtype)
            if pos0:
                head = qkv[:pos0].clone()
                kernels.qk_norm_rope_write(head, batch(0, pos0), None, None, 1e-6, None, 0, heads, kv_heads, dim, vdim, view)
            tail = qkv[pos0:].clone()
            kernels.qk_norm_rope_write(tail, batch(pos0, new), None, None, 1e-6, None, 0, heads, kv_heads, dim, vdim, view)
            out = kernels.sink_attention(tail, batch(pos0, new), heads, kv_heads, dim, vdim, 1.0, None, sinks, view)
            got = out[-1].float().cpu().view(heads, vdim)
            assert not torch.isnan(got).any()
            rep = heads // kv_heads
            if far >= start:                     # exp(36) against ones: the others' weight is below 1e-14
                want = v_all[far].to(dtype).float().view(kv_heads, vdim).repeat_interleave(rep, 0)
            else:
                seen = v_all[start:last + 1].to(dtype).float()
                want = (seen.sum(0) / (seen.shape[0] + 1)).view(kv_heads, vdim).repeat_interleave(rep, 0)
            assert torch.allclose(got, want, atol=tol), (pos0, new, far)


def test_one_key_carries_the_weight_inside_its_window_only():
    check_one_key_inside_the_window_only(TorchKernels(), "cpu")


def check_state_space_keeps_a_far_token(kernels, device, dtype=torch.float32):
    """A decay of almost one and a single token with a large step: what that token wrote into the state is read back
    200 tokens later, after portions of many sizes and single tokens, and is gone from a request that takes the slot
    over afterwards."""
    from types import SimpleNamespace

    heads, vdim, state, groups, taps = 2, 4, 3, 1, 3
    inner, GN = heads * vdim, groups * state
    C = inner + 2 * GN
    f32 = dict(dtype=torch.float32, device=device)
    conv_w = torch.zeros(C, taps, **f32)
    conv_w[:, -1] = 1.0                                          # the convolution hands the current token through
    conv_b = torch.zeros(C, **f32)
    rate = torch.tensor([1e-4, 50.0], **f32)                     # head 0 keeps, head 1 forgets at once
    zero = torch.zeros(heads, **f32)
    view = MatrixState(heads, state, vdim, C, taps).view(
        {"state": torch.full((3, heads, state, vdim), float("nan"), **f32),
         "tail": torch.full((3, taps - 1, C), float("nan"), device=device, dtype=dtype)},
        slots=torch.tensor([1], dtype=torch.int32, device=device), slot_list=[1])

    def run(proj, pos0):
        n = proj.shape[0]
        batch = SimpleNamespace(seg_lens=[n], seg_slot_list=[1], cu_seqlens=torch.tensor([0, n], dtype=torch.int32, device=device),
                                seg_of_token=torch.zeros(n, dtype=torch.int32, device=device), num_segments=1, max_seg_len=n,
                                num_tokens=n)
        return kernels.state_space(proj.to(device, dtype), conv_w, conv_b, zero, rate, zero, torch.ones(inner, **f32), 1e-12,
                                   heads, vdim, state, groups, 1, batch, view)

    def fresh():
        view.state[1].zero_()
        view.tail[1].zero_()

    silu_inv = 5.0                                               # silu(5) = 4.9665...: the same in every row that is set
    rows = torch.zeros(230, 2 * inner + 2 * GN + heads)
    rows[:, :inner] = 3.0                                        # the gate is open everywhere
    rows[:, 2 * inner + 2 * GN:] = -30.0                         # step sizes of almost nothing ...
    rows[7, 2 * inner + 2 * GN:] = 2.0                           # ... but at token 7, which writes B x^T
    rows[7, inner:2 * inner] = silu_inv
    rows[7, 2 * inner:2 * inner + GN] = silu_inv
    rows[207, 2 * inner + GN:] = silu_inv                        # token 207 reads with C
    fresh()
    outs, at = [], 0
    for n in [5, 2, 9, 1, 1, 17, 3, 1, 64, 70, 1, 1, 2, 31, 22]:
        outs.append(run(rows[at:at + n], at).float().cpu())
        at += n
    out = torch.cat(outs)
    assert at == 230 and not torch.isnan(out).any()
    # head 0 still holds what token 7 wrote; the norm over the whole row leaves its sign and share: head 1 reads nothing
    assert float(out[207, :vdim].abs().min()) > 0.5 and float(out[207, vdim:].abs().max()) < 1e-3
    assert float(out[206].abs().max()) < 1e-3 and float(out[208].abs().max()) < 1e-3
    # the same rows from token 8 on in a slot that was cleared: nothing to read
    fresh()
    again = run(rows[8:], 8).float().cpu()
    assert float(again[207 - 8].abs().max()) < 1e-3


def test_state_space_keeps_a_far_token():
    check_state_space_keeps_a_far_token(TorchKernels(), "cpu")


def test_the_plain_mechanisms_by_hand():
    """The oracle's own functions against numbers worked out by hand."""
    D = torch.float64
    # Dynamic Tanh: no statistic of the row, one slope
    w = {"n": torch.tensor([2.0, 1.0], dtype=D), "n.b": torch.tensor([0.5, -1.0], dtype=D), "n.alpha": torch.tensor(0.5, dtype=D)}
    out = plain_sezanex.dyt(torch.tensor([[2.0, -4.0]], dtype=D), w, "n")
    assert torch.allclose(out, torch.tensor([[2 * math.tanh(1.0) + 0.5, math.tanh(-2.0) - 1.0]], dtype=D))
    # RMS norm: eps inside the root
    x = torch.tensor([[3.0, 4.0]], dtype=D)
    assert torch.allclose(plain_sezanex.rms(x, 0.5), x / math.sqrt(12.5 + 0.5))
    # blended frequencies: 8 dims, base 16, original length 2 pi * 4: the pair that turns t times has index 4 ln(4 / t) / ln 16
    rot = {"dims": 8, "base": 16.0, "scaling": {"factor": 4.0, "original": 8 * math.pi, "fast": 4.0, "slow": 0.25}}
    freq, amp = plain_sezanex.yarn_frequencies(rot)
    # index(fast) = 0 -> low 0; index(slow) = 4 ln 16 / ln 16 = 4 -> high 4; ramp 0, 1/4, 1/2, 3/4
    plain = [16.0 ** (-2 * i / 8) for i in range(4)]
    want = [plain[0], plain[1] * (0.25 / 4 + 0.75), plain[2] * (0.5 / 4 + 0.5), plain[3] * (0.75 / 4 + 0.25)]
    assert torch.allclose(freq, torch.tensor(want, dtype=D)) and abs(amp - (0.1 * math.log(4.0) + 1)) < 1e-15
    # rotation: element i pairs with i + dims/2, elements past dims pass unchanged, position 0 only gets the amplitude
    v = torch.arange(1.0, 13.0, dtype=D).view(2, 1, 6)
    out = plain_sezanex.rotate(v, torch.tensor([0, 5]), {"dims": 4, "base": 100.0})
    assert torch.equal(out[0], v[0]) and torch.equal(out[..., 4:], v[..., 4:])
    a = 5 * 100.0 ** (-2 / 4)
    assert abs(float(out[1, 0, 1]) - (8 * math.cos(a) - 10 * math.sin(a))) < 1e-9
    assert abs(float(out[1, 0, 3]) - (10 * math.cos(a) + 8 * math.sin(a))) < 1e-9
    # the constant in the denominator takes weight from the keys and gives it to nothing; the norm runs over all heads at once
    m = {"heads": 2, "kv_heads": 1, "dim": 1, "vdim": 1, "mask": {"size": 2}, "scale": 1.0}
    one = torch.ones(1, 1, dtype=D)
    aw = {"q": torch.tensor([[3.0], [4.0]], dtype=D), "k": torch.zeros(1, 1, dtype=D), "v": one,
          "q.norm": torch.ones(2, dtype=D), "k.norm": torch.ones(1, dtype=D), "o": torch.tensor([[1.0, 10.0]], dtype=D)}
    out = plain_sezanex.window_attention(torch.tensor([[3.0], [6.0], [12.0]], dtype=D), aw, "", m, 1e-12)
    # all keys are zero, so every score is 0 = the constant's: one key -> 1/2, two keys -> 1/3 each; the window holds two
    assert torch.allclose(out, torch.tensor([[11 * 3.0 / 2], [11 * (3.0 + 6.0) / 3], [11 * (6.0 + 12.0) / 3]], dtype=D))
    q = plain_sezanex.rms(torch.tensor([[3.0, 4.0]], dtype=D), 0.0)          # both heads share one root mean square
    assert torch.allclose(q, torch.tensor([[3.0, 4.0]], dtype=D) / math.sqrt(12.5))
    # the convolution: the last column is the current token's, zeros before the start
    c = plain_sezanex.causal_conv_silu(torch.tensor([[1.0], [2.0]], dtype=D), torch.tensor([[10.0, 3.0]], dtype=D),
                                       torch.tensor([0.25], dtype=D))
    s = lambda z: z / (1 + math.exp(-z))
    assert torch.allclose(c, torch.tensor([[s(3.25)], [s(10 + 6 + 0.25)]], dtype=D))
    # the state-space mixer: one head, a state of one number, no convolution to speak of (one tap of 1)
    mm = {"heads": 1, "vdim": 1, "state": 1, "groups": 1, "norm_groups": 1, "conv": 1}
    sw = {"in": torch.tensor([[1.0], [1.0], [1.0], [1.0], [1.0]], dtype=D), "conv": torch.ones(3, 1, dtype=D),
          "conv.b": torch.zeros(3, dtype=D), "dt_bias": torch.tensor([0.5], dtype=D), "A_log": torch.tensor([math.log(2.0)], dtype=D),
          "D": torch.tensor([0.1], dtype=D), "norm": torch.ones(1, dtype=D), "o": one}
    h = torch.tensor([[1.0], [2.0]], dtype=D)
    dt1, dt2 = math.log1p(math.exp(1.5)), math.log1p(math.exp(2.5))
    S1 = dt1 * s(1.0) * s(1.0)
    S2 = math.exp(-2.0 * dt2) * S1 + dt2 * s(2.0) * s(2.0)
    y1, y2 = S1 * s(1.0) + 0.1 * s(1.0), S2 * s(2.0) + 0.1 * s(2.0)
    got = plain_sezanex.mamba2_mixer(h, sw, "", mm, 0.0)
    assert y1 > 0 and y2 > 0 and torch.allclose(got, torch.ones(2, 1, dtype=D))      # one element: the norm leaves its sign
    sw["norm"] = torch.tensor([1.0, 1.0], dtype=D)
    mm2 = dict(mm, vdim=2)
    sw2 = dict(sw, **{"in": torch.tensor([[1.0], [1.0], [1.0], [0.5], [1.0], [1.0], [1.0]], dtype=D), "conv": torch.ones(4, 1, dtype=D),
                      "conv.b": torch.zeros(4, dtype=D), "o": torch.eye(2, dtype=D)})
    got = plain_sezanex.mamba2_mixer(h[:1], sw2, "", mm2, 0.0)
    ya, yb = (dt1 * s(1.0) * s(1.0) + 0.1) * s(1.0) * s(1.0), (dt1 * s(1.0) * s(1.0) + 0.1) * s(0.5) * s(1.0)
    r = math.sqrt((ya * ya + yb * yb) / 2)
    assert torch.allclose(got, torch.tensor([[ya / r, yb / r]], dtype=D))            # gate first, then the norm
    # experts: sigmoid scores, not renormalised, on the expert's INPUT
    f = {"router": {"experts": 3, "top": 2}}
    ew = {"router": torch.tensor([[1.0], [-1.0], [0.5]], dtype=D)}
    for e in range(3):
        ew[f"e{e}.gate"], ew[f"e{e}.up"], ew[f"e{e}.down"] = one * (e + 1), one, one
    got = plain_sezanex.sigmoid_experts(torch.tensor([[2.0]], dtype=D), ew, "", f)
    s0, s2 = 1 / (1 + math.exp(-2.0)), 1 / (1 + math.exp(-1.0))                       # experts 0 and 2 lead
    want = s(1 * s0 * 2.0) * (s0 * 2.0) + s(3 * s2 * 2.0) * (s2 * 2.0)
    assert abs(float(got) - want) < 1e-12
    # the dense feed-forward: the erf GELU
    dw = {"up": torch.tensor([[1.0]], dtype=D), "down": torch.tensor([[2.0]], dtype=D)}
    assert abs(float(plain_sezanex.dense_ff(torch.tensor([[0.7]], dtype=D), dw, "")) - 0.7 * (1 + math.erf(0.7 / math.sqrt(2)))) < 1e-12
    # the order of layers: a loop over layers 1 and 2 that runs twice; a pass starts at layer 1 both times
    order = plain_sezanex.layer_order({"layers": [0, 1, 2, 3], "loop": {"start": 1, "stop": 3, "times": 2}})
    assert order == [(0, False), (1, True), (2, False), (1, True), (2, False), (3, False)]


def test_trace_replay_of_a_sezanex_folder(tmp_path):
    folder = cases.write_folder(str(tmp_path / "m"), cases.ODD, seed=5)
    cfg, w = cases.read_folder(folder)
    toks = helpers.random_tokens(cfg["vocab"], 15, 9)
    other = helpers.random_tokens(cfg["vocab"], 6, 10)
    ref, ref_other = _plain(cfg, w, toks), _plain(cfg, w, other)
    lines = [{"step": 0, "entries": [{"id": "a", "tokens": toks[:9], "want": [0, 8]}], "end": []},
             {"step": 1, "entries": [{"id": "a", "tokens": toks[9:11], "want": []}, {"id": "b", "tokens": other[:4], "want": [3]}], "end": []},
             {"step": 2, "entries": [{"id": "b", "tokens": other[4:], "want": [1]}, {"id": "a", "tokens": toks[11:], "want": [3]}],
              "end": ["a", "b"]}]
    log = io.StringIO()
    run_trace(folder, "float32", str(tmp_path / "out"), 128, [json.dumps(l) for l in lines], log=log, device="cpu",
              kernels=TorchKernels(), page_size=16)
    assert log.getvalue().split() == ["done", "0", "done", "1", "done", "2"]
    s0 = np.fromfile(tmp_path / "out" / "0.f32", dtype="<f4").reshape(2, cfg["vocab"])
    s1 = np.fromfile(tmp_path / "out" / "1.f32", dtype="<f4").reshape(1, cfg["vocab"])
    s2 = np.fromfile(tmp_path / "out" / "2.f32", dtype="<f4").reshape(2, cfg["vocab"])
    scale = float(ref.abs().max())
    assert np.abs(s0 - ref[[0, 8]].numpy()).max() < 2e-5 * scale and np.abs(s1 - ref_other[[3]].numpy()).max() < 2e-5 * scale
    assert np.abs(s2[0] - ref_other[5].numpy()).max() < 2e-5 * scale and np.abs(s2[1] - ref[14].numpy()).max() < 2e-5 * scale


def test_greedy_generation_through_the_scheduler_under_page_pressure(tmp_path):
    from tt_transformers_b200.engine.llm import from_pretrained

    folder = cases.write_folder(str(tmp_path / "g"), cases.PLAIN, seed=7)
    cfg, w = cases.read_folder(folder)
    prompts = [helpers.random_tokens(cfg["vocab"], n, 80 + n) for n in (4, 13, 21)]

    def plain_greedy(prompt, new):
        toks = list(prompt)
        for _ in range(new):
            toks.append(int(_plain(cfg, w, toks)[-1].argmax()))
        return toks[len(prompt):]

    expect = [plain_greedy(p, 6) for p in prompts]
    # 7 pages of 8 tokens for requests that end at 10, 19 and 27 tokens: they cannot all stay, one gives way and is
    # recomputed from a zeroed state
    llm = from_pretrained(folder, dtype="float32", page_size=8, num_pages=7, max_batch_size=3, max_seq_len=64,
                          max_step_tokens=16, max_chunk_tokens=8, device="cpu", kernels=TorchKernels())
    assert llm.generate(prompts, max_new_tokens=6) == expect
    llm.engine.cache.audit()
    assert llm.engine.cache.free_pages() == 7
