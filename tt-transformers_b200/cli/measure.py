"""Measuring code shared by bench.py and the benchmark command line.

Every figure comes from the engine that generation uses: `build_engine`, `Engine.step`,
`Engine.decode_steps`, `LLM.add_request/step`. Times are CUDA events on the launching stream after
warm-up steps, wall clock only where the host is part of what is measured (end to end, time to first
token). Roofline fractions divide by the peaks in MEASURED_PEAKS.json at the repository's root when
that file is there ("measured"), else by fixed fallback figures ("fallback").

The reference reports the same kinds of numbers for its own hardware: time to first token, tokens a
second per user and in total (examples/common/run_helpers.py:86-101), and a teacher-forced accuracy
against a float32 run (examples/common/run_helpers.py:201-289).
"""

from __future__ import annotations

import atexit
import json
import os
import statistics
import subprocess
import threading
import time
from typing import Dict, List, Optional

import torch

from .common import RANDOM_MODELS

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
MODEL_NAMES = {"1b": "llama-3.2-1b", "3b": "llama-3.2-3b", "8b": "llama-3.1-8b"}
PAGE = 16
PREFILL_TOKENS = 2048
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def model_config(name: str) -> dict:
    return dict(RANDOM_MODELS[MODEL_NAMES.get(name, name)])


def peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.isfile(path):
        with open(path) as f:
            data = json.load(f)
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {**FALLBACK_PEAKS, "bf16_tflops_sustained": FALLBACK_PEAKS["bf16_tflops"], "source": "fallback"}


def fp32_pipe_tflops(device: int = 0) -> float:
    """What the float32 multiply-add pipe can do: SMs x 128 lanes x 2 FLOPs x the highest SM clock (nominal, not measured)."""
    props = torch.cuda.get_device_properties(device)
    mhz = getattr(props, "clock_rate", 0) / 1e3 or 1965.0
    return props.multi_processor_count * 128 * 2 * mhz * 1e6 / 1e12


class ClockSampler:
    """nvidia-smi in the background for the whole run (reading only); a timed region keeps the samples that
    arrived while it ran, or, if the region was shorter than the sampling period, the sample nearest to it."""

    QUERY = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, period_ms: int = 50):
        self.samples = []                   # (arrival time, SM MHz, max SM MHz, active reasons)
        self.proc = None
        self.summary = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", "0", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", str(period_ms)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        atexit.register(self.stop)          # whatever way the run ends, the child does not outlive it
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 6:
                continue
            try:
                clock, max_clock = float(parts[0]), float(parts[1])
            except ValueError:
                continue
            reasons = [n for n, flag in zip(self.NAMES, parts[2:6]) if flag.lower().startswith("active")]
            self.samples.append((time.perf_counter(), clock, max_clock, reasons))

    def wait_for_first_sample(self, timeout_s: float = 5.0):
        end = time.perf_counter() + timeout_s
        while self.proc is not None and not self.samples and time.perf_counter() < end:
            time.sleep(0.01)

    def __enter__(self):
        self.t0 = time.perf_counter()
        return self

    def __exit__(self, *exc):
        t1 = time.perf_counter()
        self.summary = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
        if self.proc is None:
            return
        time.sleep(0.03)                    # a sample taken at the region's end may still be on its way
        inside = [x for x in self.samples if self.t0 <= x[0] <= t1 + 0.03]
        if not inside and self.samples:
            inside = [min(self.samples, key=lambda x: min(abs(x[0] - self.t0), abs(x[0] - t1)))]
        if inside:
            self.summary = {"sm_mhz": statistics.median(x[1] for x in inside), "sm_max_mhz": inside[-1][2],
                            "reasons": sorted({r for x in inside for r in x[3]})}

    def stop(self):
        if self.proc is not None and self.proc.poll() is None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()


# ---------------------------------------------------------------------------- what a step has to move and compute
def weight_bytes(cfg: dict, layers: int, elem: int = 2) -> int:
    """Every weight a decode step reads once (the embedding rows it gathers are negligible; an untied head is
    the table it multiplies by, a tied one the embedding table)."""
    d, inter, vocab = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    heads, kv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    per_layer = (heads + 2 * kv) * hd * d + heads * hd * d + 3 * inter * d + 2 * d
    return (layers * per_layer + vocab * d + d) * elem


def cache_bytes_per_token(cfg: dict, layers: int, elem: int = 2) -> int:
    return layers * 2 * cfg["num_key_value_heads"] * cfg["head_dim"] * elem


def decode_bytes(cfg: dict, layers: int, contexts, elem: int = 2) -> int:
    """Bytes a decode step has to read: every weight once, and the cache of the live requests
    (`contexts`: tokens each of them holds)."""
    return weight_bytes(cfg, layers, elem) + sum(contexts) * cache_bytes_per_token(cfg, layers, elem)


def prefill_flops(cfg: dict, layers: int, tokens: int) -> float:
    d, inter, vocab = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    heads, kv, hd = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    linear = 2 * tokens * ((heads + 2 * kv) * hd * d + heads * hd * d + 3 * inter * d)
    attention = 2 * 2 * heads * hd * tokens * (tokens + 1) / 2      # causal QK^T and PV
    return layers * (linear + attention) + 2 * vocab * d            # plus one row of logits


def timed(fn, reps: int) -> float:
    """Milliseconds per call of fn, CUDA events around `reps` calls on the current stream."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / reps


class Prompts:
    def __init__(self, vocab: int, seed: int = 0):
        self.vocab, self.gen = vocab, torch.Generator().manual_seed(seed)

    def __call__(self, n: int) -> List[int]:
        return torch.randint(0, self.vocab, (n,), generator=self.gen).tolist()

    def length(self, low: int, high: int) -> int:
        return int(torch.randint(low, high + 1, (1,), generator=self.gen))


# ---------------------------------------------------------------------------- the engine under measurement
def make_engine(cfg: dict, *, layers: Optional[int] = None, dtype: str = "bfloat16", max_batch: int, context: int,
                pool_tokens: Optional[int] = None, step_tokens: int = PREFILL_TOKENS, seed: int = 0,
                device: str = "cuda:0", cuda_graph: bool = True, tensors: Dict[str, torch.Tensor] = None):
    """An engine of the named sizes with random weights N(0, 0.02) drawn on the GPU. `pool_tokens`: how many
    tokens the page pool holds (default max_batch * context)."""
    from ..config.engine import EngineConfig
    from ..engine.step import build_engine
    from ..weights import random_tensors

    torch.cuda.set_device(torch.device(device))
    if tensors is None:
        tensors = random_tensors(cfg, seed=seed, dtype=torch.bfloat16 if dtype == "bfloat16" else torch.float32,
                                 device=device)
    pool = pool_tokens if pool_tokens is not None else max_batch * context
    engine = build_engine(config_dict=cfg, tensors=tensors, n_layers=layers, engine_config=EngineConfig(
        dtype=dtype, page_size=PAGE, num_pages=-(-pool // PAGE) + max_batch, max_batch_size=max_batch,
        max_seq_len=context, max_step_tokens=step_tokens, max_chunk_tokens=step_tokens, cuda_graph=cuda_graph,
        device=device))
    return engine


def measure_prefill(engine, cfg: dict, layers: int, pk: dict, tokens: int = PREFILL_TOKENS, prompts: Prompts = None) -> dict:
    """One prompt of `tokens` tokens in one step, logits of its last token. Steps back to back, so that the
    host's part of a step runs under the step before; the median of three runs of five."""
    from ..engine.step import StepEntry

    prompts = prompts or Prompts(cfg["vocab_size"])
    ids = prompts(tokens)

    def once():
        engine.step([StepEntry("prefill", ids, [tokens - 1])])
        engine.finish("prefill")

    for _ in range(3):
        once()
    ms = statistics.median(timed(once, 5) for _ in range(3))
    flops = prefill_flops(cfg, layers, tokens)
    return {"value": round(tokens / ms * 1e3, 1), "tokens": tokens, "ms": round(ms, 3),
            "frac": round(flops / (ms * 1e-3) / (pk["bf16_tflops"] * 1e12), 4)}


def measure_ttft(engine, cfg: dict, prompt_tokens: int = 128, reps: int = 20, prompts: Prompts = None) -> dict:
    """Time to the first token of one short prompt arriving at an idle engine: host token ids in, the sampled
    id back on the host; wall clock, median of `reps`."""
    from ..engine.step import StepEntry

    prompts = prompts or Prompts(cfg["vocab_size"])
    ids = prompts(prompt_tokens)
    times = []
    for i in range(reps + 3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        logits = engine.step([StepEntry("ttft", ids, [prompt_tokens - 1])])
        int(engine.kernels.sample(logits)[0])            # the host has the token
        times.append((time.perf_counter() - t0) * 1e3)
        engine.finish("ttft")
    return {"prompt_tokens": prompt_tokens, "ms": round(statistics.median(times[3:]), 3)}


def fill_requests(engine, cfg: dict, batch: int, length: int, prompts: Prompts, how: str = "prefill",
                  prefix: str = "d") -> List[str]:
    """`batch` live requests that hold `length` tokens each: through the engine's own chunked prefill, or
    (`synthetic`) pages reserved and filled with random numbers, which decode timing cannot tell apart."""
    from ..engine.step import StepEntry

    ids = [f"{prefix}{i}" for i in range(batch)]
    if how == "synthetic":
        for rid in ids:
            engine.cache.admit(rid)
            engine.cache.reserve(rid, length)
            engine.cache.commit(rid, length)
        for g in engine.cache.groups:
            if g.pool is not None:
                for tensor in g.storage.values():
                    tensor.normal_(0, 1)
        return ids
    budget = engine.config.max_step_tokens
    for rid in ids:
        tokens = prompts(length)
        for i in range(0, length, budget):
            engine.step([StepEntry(rid, tokens[i:i + budget], [])])
    return ids


def measure_decode(engine, cfg: dict, layers: int, pk: dict, batch: int, context: int, steps: int, warmup: int,
                   sampler: ClockSampler = None, how: str = "prefill", prompts: Prompts = None) -> dict:
    """`steps` decode steps of `batch` requests that hold about `context` tokens each, through the engine's
    decode loop (every step takes its tokens from the step before, on the device)."""
    prompts = prompts or Prompts(cfg["vocab_size"])
    start = context - steps - warmup - 1
    ids = fill_requests(engine, cfg, batch, start, prompts, how)
    if how == "prefill":
        # Filling the cache is a burst of tensor-core work that leaves the board at its power cap with lowered
        # clocks; decoding does not keep it there. Let the clocks settle so that the timed steps measure decoding.
        torch.cuda.synchronize()
        time.sleep(0.5)
    tokens = engine.decode_steps(ids, [1] * batch, warmup)[-1]
    before = engine.kernels.launches
    clocks = {"sm_mhz": None, "sm_max_mhz": None, "reasons": []}
    if sampler is not None:
        sampler.wait_for_first_sample()
        with sampler:
            ms = timed(lambda: engine.decode_steps(ids, tokens, steps), 1) / steps
        clocks = sampler.summary
    else:
        ms = timed(lambda: engine.decode_steps(ids, tokens, steps), 1) / steps
    launches = engine.kernels.launches - before
    held = [engine.cache.length(rid) for rid in ids]
    for rid in ids:
        engine.finish(rid)
    # the cache read in the middle of the timed steps
    need = decode_bytes(cfg, layers, [n - steps // 2 for n in held])
    achieved = need / (ms * 1e-3) / 1e9
    return {"batch": batch, "context": context, "steps": steps, "ms_per_step": round(ms, 4),
            "tokens_per_s": round(batch / ms * 1e3, 1), "tokens_per_s_per_user": round(1e3 / ms, 1),
            "gpu_launches": launches, "clocks": clocks,
            "roofline": {"bound": "hbm", "bytes_per_step": need, "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4), "peaks": pk["source"]}}


def measure_e2e(llm, cfg: dict, batch: int, context: int, steps: int, warmup: int, prompts: Prompts = None,
                how: str = "prefill") -> dict:
    """The same decode steps through the Python entry point: host token ids in, sampled ids back on the host
    every step; wall clock around synchronised steps."""
    from ..sampling import SamplingParams

    engine = llm.engine
    prompts = prompts or Prompts(cfg["vocab_size"])
    params = SamplingParams(temperature=0.0, max_new_tokens=1 << 30, ignore_eos=True)
    # Requests whose prompts are done decode while the others' prompts are still being computed, one token for
    # every later prompt portion: leave room for that, so that nobody reaches the context limit inside the
    # timed region.
    length = context - steps - warmup - 2 - batch * (context // engine.config.max_step_tokens + 1)
    if how == "synthetic":
        for _ in range(batch):
            llm.add_request(prompts(length), params)
        sched = llm._scheduler
        for r in list(sched.waiting):     # the prompts' last token goes through the engine; the rest is filled
            sched.waiting.remove(r)
            engine.cache.admit(r.request_id)
            engine.cache.reserve(r.request_id, length - 1)
            engine.cache.commit(r.request_id, length - 1)
            r.num_computed = length - 1
            sched.running.append(r)
    else:
        for _ in range(batch):
            llm.add_request(prompts(length), params)
        while any(r.num_computed < len(r.prompt) for r in llm._scheduler.running) or llm._scheduler.waiting:
            llm.step()
    for _ in range(warmup):
        llm.step()
    torch.cuda.synchronize()
    h2d, d2h = engine.h2d_bytes, llm.d2h_bytes
    t0 = time.perf_counter()
    for _ in range(steps):
        llm.step()
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) * 1e3 / steps
    return {"value": round(batch / ms * 1e3, 1), "unit": "tokens/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": (engine.h2d_bytes - h2d) // steps, "d2h_bytes_per_step": (llm.d2h_bytes - d2h) // steps}


# ---------------------------------------------------------------------------- the scheduler under mixed load
def run_mixed(llm, cfg: dict, layers: int, pk: dict, requests: int = 32, prompt_low: int = 128, prompt_high: int = 2048,
              new_tokens: int = 256, seed: int = 0, sampler: ClockSampler = None) -> dict:
    """`requests` prompts of lengths uniform in [prompt_low, prompt_high] arrive together; every one decodes
    `new_tokens` tokens; the scheduler cuts the prompts under its token budget beside the decoding requests.
    Reports tokens a second over the whole run, mean time to first token, decoded tokens a second per user,
    and for the steps in which every live request decodes, the share of the HBM peak that (weights + the live
    requests' cache) a step stands for. One pass warms up (graphs are captured), the second is measured."""
    from ..sampling import SamplingParams

    engine = llm.engine
    params = SamplingParams(temperature=0.0, max_new_tokens=new_tokens, ignore_eos=True)
    result = {}
    for run in ("warm-up", "measured"):
        prompts = Prompts(cfg["vocab_size"], seed)
        lengths = [prompts.length(prompt_low, prompt_high) for _ in range(requests)]
        reqs = [llm.add_request(prompts(n), params) for n in lengths]
        first, last = {}, {}
        decode_only = []                 # (seconds, bytes) of steps in which every live request decodes
        if sampler is not None and run == "measured":
            sampler.wait_for_first_sample()
            sampler.__enter__()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        steps = 0
        while llm.has_unfinished():
            sched = llm._scheduler
            all_decoding = (not sched.waiting and sched.running
                            and all(r.num_computed >= len(r.prompt) for r in sched.running))
            contexts = [r.num_tokens for r in sched.running] if all_decoding else None
            t = time.perf_counter()
            llm.step()
            now = time.perf_counter()
            steps += 1
            if contexts is not None:
                decode_only.append((now - t, decode_bytes(cfg, layers, contexts)))
            for r in reqs:
                if r.output and r.request_id not in first:
                    first[r.request_id] = now - t0
                if r.finish_reason is not None and r.request_id not in last:
                    last[r.request_id] = now - t0
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        if sampler is not None and run == "measured":
            sampler.__exit__(None, None, None)
        generated = sum(len(r.output) for r in reqs)
        per_user = [(len(r.output) - 1) / (last[r.request_id] - first[r.request_id]) for r in reqs
                    if len(r.output) > 1 and last[r.request_id] > first[r.request_id]]
        # the look-ahead launches a step while the host waits for the one before: single step times are not
        # meaningful, their sum over a run of decode-only steps is
        seconds = sum(s for s, _ in decode_only)
        moved = sum(b for _, b in decode_only)
        result = {
            "requests": requests, "prompt_tokens": sum(lengths), "generated_tokens": generated, "steps": steps,
            "wall_s": round(wall, 4),
            "tokens_per_s": round(generated / wall, 1),
            "tokens_per_s_with_prompts": round((generated + sum(lengths)) / wall, 1),
            "mean_ttft_ms": round(1e3 * statistics.mean(first.values()), 2),
            "max_ttft_ms": round(1e3 * max(first.values()), 2),
            "decode_tokens_per_s_per_user": round(statistics.mean(per_user), 1),
            "preemptions": llm._scheduler.preemptions if llm._scheduler else 0,
            "decode_only_steps": len(decode_only),
            "roofline": {"bound": "hbm", "what": "steps in which every live request decodes",
                         "achieved": round(moved / seconds / 1e9, 1) if seconds else None, "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(moved / seconds / 1e9 / pk["hbm_gbs"], 4) if seconds else None,
                         "peaks": pk["source"]},
            "clocks": sampler.summary if sampler is not None else None,
        }
    return result


# ---------------------------------------------------------------------------- float32 logits against the plain implementation
def load_plain():
    """The plain implementation lives with the tests (tests/plain_llama.py): it shares no code with the package
    and is loaded from there by path."""
    import importlib.util

    path = os.path.join(ROOT, "tests", "plain_llama.py")
    if not os.path.isfile(path):
        raise FileNotFoundError(f"{path}: the plain implementation that token-match compares with is not there")
    spec = importlib.util.spec_from_file_location("plain_llama", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def _cuttings(requests: Dict[str, List[int]], tail: int = 32):
    """The four ways of cutting requests into steps: whole, last tokens one by one, portions of changing size,
    mixed (up to four live, portions beside decoded tokens)."""
    whole = [{"entries": [(rid, toks, list(range(len(toks))))], "end": [rid]} for rid, toks in requests.items()]
    decode_tail = []
    for rid, toks in requests.items():
        head = max(1, len(toks) - tail)
        decode_tail.append({"entries": [(rid, toks[:head], list(range(head)))], "end": [rid] if head == len(toks) else []})
        for i in range(head, len(toks)):
            decode_tail.append({"entries": [(rid, [toks[i]], [0])], "end": [rid] if i == len(toks) - 1 else []})
    portions, sizes = [], (7, 5, 3, 2, 2, 11, 4, 2, 16, 9)
    for rid, toks in requests.items():
        i, k = 0, 0
        while i < len(toks):
            n = min(sizes[k % len(sizes)], len(toks) - i)
            portions.append({"entries": [(rid, toks[i:i + n], list(range(n)))], "end": [rid] if i + n == len(toks) else []})
            i, k = i + n, k + 1
    mixed, at, k = [], {rid: 0 for rid in requests}, 0
    while at:
        entries, end = [], []
        for j, rid in enumerate(list(at)):
            toks, i = requests[rid], at[rid]
            if i >= len(toks) - 8:
                n = 1                                       # the last tokens of a request one by one
            else:
                n = min(sizes[(k + 3 * j) % len(sizes)], len(toks) - 8 - i)
            entries.append((rid, toks[i:i + n], list(range(n))))
            at[rid] = i + n
            if at[rid] == len(toks):
                end.append(rid)
                del at[rid]
        mixed.append({"entries": entries, "end": end})
        k += 1
    return {"whole": whole, "decode_tail": decode_tail, "portions": portions, "mixed": mixed}


def run_token_match(cfg: dict, *, layers: Optional[int] = None, prompt_lengths=(96, 61), seed: int = 0,
                    dtype: str = "float32", device: str = "cuda:0") -> dict:
    """The engine in `dtype` against the plain float32 implementation on the same random weights, in the four
    ways of cutting: per mode the largest relative error of the logits (max |engine - plain| / max |plain|, over
    every position of every prompt) and the share of positions whose best token agrees."""
    from ..engine.step import StepEntry
    from ..weights import random_tensors

    plain = load_plain()
    layers = layers or cfg["num_hidden_layers"]
    cfg = dict(cfg, num_hidden_layers=layers)
    weights = random_tensors(cfg, seed=seed, dtype=torch.float32, device="cpu")
    prompts = Prompts(cfg["vocab_size"], seed + 1)
    requests = {f"p{i}": prompts(n) for i, n in enumerate(prompt_lengths)}
    t0 = time.perf_counter()
    with torch.no_grad():
        ref = {rid: plain.forward(cfg, weights, toks) for rid, toks in requests.items()}
    plain_s = time.perf_counter() - t0
    engine = make_engine(cfg, dtype=dtype, max_batch=4, context=max(prompt_lengths) + PAGE, cuda_graph=True,
                         tensors=weights, device=device)
    del weights
    modes = {}
    for mode, steps in _cuttings(requests).items():
        got: Dict[str, list] = {}
        for step in steps:
            logits = engine.step([StepEntry(rid, toks, want) for rid, toks, want in step["entries"]]).float().cpu()
            row = 0
            for rid, _, want in step["entries"]:
                for _ in want:
                    got.setdefault(rid, []).append(logits[row])
                    row += 1
            for rid in step["end"]:
                engine.finish(rid)
        engine.kernels.check_status()
        worst, agree, count = 0.0, 0, 0
        for rid in requests:
            mine = torch.stack(got[rid])
            worst = max(worst, float((mine - ref[rid]).abs().max() / ref[rid].abs().max()))
            agree += int((mine.argmax(-1) == ref[rid].argmax(-1)).sum())
            count += mine.shape[0]
        modes[mode] = {"max_relative_error": worst, "argmax_agreement": agree / count, "positions": count}
    engine.close()
    return {"dtype": dtype, "layers": layers, "prompt_lengths": list(prompt_lengths), "plain_seconds": round(plain_s, 2),
            "modes": modes, "max_relative_error": max(m["max_relative_error"] for m in modes.values()),
            "argmax_agreement": min(m["argmax_agreement"] for m in modes.values())}


# ---------------------------------------------------------------------------- a design beside its closest dense model
class KernelTimer:
    """CUDA events around the calls of named entries of an engine's kernel table (outermost calls only), for
    steps that run eagerly. The device is kept busy ahead of a step (`hold`), so that the host's launch gaps
    do not lie between a pair of events."""

    def __init__(self, kernels, names):
        self.kernels, self.names, self.records, self.depth = kernels, names, [], 0
        self._originals = {}

    def __enter__(self):
        for name in self.names:
            original = getattr(self.kernels, name)
            self._originals[name] = original

            def wrapped(*args, _original=original, _name=name, **kwargs):
                if self.depth:
                    return _original(*args, **kwargs)
                self.depth += 1
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                try:
                    return _original(*args, **kwargs)
                finally:
                    end.record()
                    self.records.append((_name, start, end))
                    self.depth -= 1

            setattr(self.kernels, name, wrapped)
        return self

    def __exit__(self, *exc):
        for name in self.names:
            delattr(self.kernels, name)               # the instance attribute goes, the class's method shows again
        return False

    @staticmethod
    def hold(ms: float = 5.0):
        torch.cuda._sleep(int(ms * 1.8e6))            # the device spins while the host queues the step

    def totals(self) -> Dict[str, float]:
        torch.cuda.synchronize()
        out: Dict[str, float] = {}
        for name, start, end in self.records:
            out[name] = out.get(name, 0.0) + start.elapsed_time(end) * 1e3
        self.records = []
        return out                                     # microseconds per name


_TIMED = {"Bozavik": ["add_layernorm", "latent_prepare", "heads_linear", "_latent_attention", "latent_out", "gate_heads", "route_top",
                      "routed_experts", "linear"],
          "Pedazen": ["stream_add_norm", "lightning_attention", "gated_rmsnorm", "qk_norm_rope_write", "sink_attention",
                      "causal_conv", "heads_linear", "gated_recurrence", "recurrent_token", "mean_rmsnorm_pair", "route_grouped", "plain_experts",
                      "glu_activation", "linear"],
          "Sezanex": ["add_dyntanh", "state_space", "qk_norm_rope_write", "sink_attention", "route_top", "input_weighted_experts",
                      "activation", "concat_cast", "linear"],
          "Bufolorn": ["add_layernorm_sum", "token_shift", "heads_linear", "lowrank_expand", "shifted_state", "short_conv_silu",
                       "delta_rule", "qk_norm_rope_write", "sink_attention", "latent_prepare", "_latent_attention", "latent_out",
                       "gate_heads", "route_corrected", "routed_experts", "glu_activation", "linear"],
          "Llama": ["add_rmsnorm", "rope_kv_write", "fused_qkv_rope", "paged_attention", "linear_swiglu", "linear"]}


def _kernel_work(cfg: dict, tokens: int, contexts: List[int], new_per_request: int) -> Dict[str, dict]:
    """Algorithmic FLOPs and bytes per step of the kernels that are the design's own, per layer summed over the
    layers: {kernel name: {"flops": .., "bytes": ..}}. contexts: tokens each request holds after the step."""
    work: Dict[str, dict] = {}

    def add(name, flops, nbytes):
        w = work.setdefault(name, {"flops": 0.0, "bytes": 0.0})
        w["flops"] += flops
        w["bytes"] += nbytes

    if cfg.get("architecture") == "Bozavik":
        width = cfg["width"]
        for layer in cfg["layers"]:
            m, f = layer["mixer"], layer["mlp"]
            dk = m["kv_rank"] + m.get("rot_dim", 0)
            pairs = sum(n * new_per_request - new_per_request * (new_per_request - 1) / 2 for n in contexts)   # visible (query, key) pairs
            add("latent_attention", 2 * m["heads"] * pairs * (dk + m["kv_rank"]),
                2 * (sum(contexts) * dk + 2 * tokens * m["heads"] * m["kv_rank"]))
            add("add_layernorm", 0, 2 * tokens * width * (4 + 4 + 2 + 2))
            add("latent_prepare", 0, tokens * (4 * (m["q_rank"] + dk) + 2 * (m["q_rank"] + dk)))
            if f:
                top, ff, experts = f["router"]["top"], f["expert"]["ff"], f["router"]["experts"]
                used = min(experts, tokens * top)
                sff = (f.get("shared") or {}).get("ff", 0)          # the shared expert runs inside the same call
                add("routed_experts", 2 * tokens * 3 * (top * ff + sff) * width,
                    2 * (used * ff + sff) * 3 * width + tokens * width * (2 + 4))
    elif cfg.get("architecture") == "Pedazen":
        width = cfg["width"]
        loop = cfg.get("loop")
        runs = [1 + ((loop["times"] - 1) if loop and loop["start"] <= i < loop["stop"] else 0) for i in range(len(cfg["layers"]))]
        for layer, times in zip(cfg["layers"], runs):
            m, f = layer["mixer"], layer["mlp"]
            for _ in range(times):
                add("stream_add_norm", 0, tokens * width * (4 + 4 + 4 + 4 + 2))            # stream in and out, two outputs in, h out
                if layer["type"] == "lightning":
                    H, D, V = m["heads"], m["dim"], m["vdim"]
                    # the recurrence costs 4 D V flops a token and head however it is cut; q, k, v in, o out, the state in and out
                    add("lightning_attention", 4.0 * tokens * H * D * V,
                        tokens * H * ((2 * D + V) * 2 + V * 4) + 2 * len(contexts) * H * D * V * 4)
                    add("gated_rmsnorm", 0, tokens * H * V * (4 + 2 + 2))
                else:
                    a, r = m["left"], m["right"]
                    H, G, D, V, C = a["heads"], a["kv_heads"], a["dim"], a["vdim"], r["width"]
                    n = a["mask"]["size"]
                    seen = []                                   # keys that the step's queries see, summed over the queries
                    for ctx in contexts:
                        for pos in range(ctx - new_per_request, ctx):
                            seen.append(pos % n + 1)
                    keys_read = sum(min(ctx, max(seen[i * new_per_request:(i + 1) * new_per_request]) + new_per_request)
                                    for i, ctx in enumerate(contexts))
                    add("sink_attention", 2.0 * H * sum(seen) * (D + V), 2 * (keys_read * G * (D + V) + tokens * H * (D + V)))
                    add("qk_norm_rope_write", 0, tokens * ((H + G) * D * 2 * 2 + G * (D + V) * 2 + G * V * 2))
                    add("causal_conv", 0, tokens * C * 2 * 2)
                    add("gated_recurrence", 0, tokens * C * (8 + 2 + 2 + 2))
                    add("heads_linear", 2.0 * tokens * 2 * C * (C // r["blocks"]), tokens * C * (2 + 8) + 2 * C * (C // r["blocks"]) * 2)
                    add("mean_rmsnorm_pair", 0, tokens * width * (2 + 2 + 4))
                if f and f["kind"] == "moe":
                    top, ff, experts = f["router"]["top"], f["expert"]["ff"], f["router"]["experts"]
                    used = min(experts, tokens * top)
                    add("plain_experts", 2.0 * tokens * 2 * top * ff * width, 2 * used * ff * 2 * width + tokens * width * (2 + 4))
                    add("route_grouped", 2.0 * tokens * experts * width, tokens * width * 2 + experts * width * 4)
    elif cfg.get("architecture") == "Bufolorn":
        width = cfg["width"]
        segs = len(contexts)
        for layer in cfg["layers"]:
            m, f = layer["mixer"], layer["mlp"]
            # the stream in and out, the layer's outputs in (two or three of them), h out
            add("add_layernorm_sum", 0, tokens * width * (4 + 4 + 2 + (2 if layer["type"] == "parallel" else 0) + (3 if f else 0) + 2))
            if layer["type"] == "parallel":
                a, r = m["left"], m["right"]
                H, G, D, V = a["heads"], a["kv_heads"], a["dim"], a["vdim"]
                pairs = sum(n * new_per_request - new_per_request * (new_per_request - 1) / 2 for n in contexts)
                add("sink_attention", 2.0 * H * pairs * (D + V), 2 * (sum(contexts) * G * (D + V) + tokens * H * (D + V)))
                add("qk_norm_rope_write", 0, tokens * ((H + G) * D * 2 * 2 + G * (D + V) * 2 + G * V * 2))
                SH, SD = r["heads"], r["dim"]
                # per token and head: the read with the bonus (2 D^2) and the decayed update (2 D^2), however it is cut;
                # r, k, v, the gate and the decays in, the output out, the state in and out
                add("shifted_state", 4.0 * tokens * SH * SD * SD, tokens * SH * SD * (4 * 2 + 4 + 2) + 2 * segs * SH * SD * SD * 4)
                work["shifted_state"]["fp32_flops"] = work["shifted_state"].get("fp32_flops", 0.0) + 4.0 * tokens * SH * SD * SD
                add("token_shift", 0, tokens * width * (2 + 5 * 2))
            elif layer["type"] == "channel_delta":
                H, G, D, V = m["heads"], m["kv_heads"], m["dim"], m["vdim"]
                C = 2 * G * D + H * V
                # per token and head: decay (D V), S^T k (2 D V), the update (2 D V), S^T q (2 D V)
                add("delta_rule", 7.0 * tokens * H * D * V, tokens * (C * 2 + H * D * 4 + H * V * 4 + H * V * 2) + 2 * segs * H * D * V * 4)
                work["delta_rule"]["fp32_flops"] = work["delta_rule"].get("fp32_flops", 0.0) + 7.0 * tokens * H * D * V
                add("short_conv_silu", 0, tokens * C * 2 * 2)
            else:
                dk = m["kv_rank"] + m.get("rot_dim", 0)
                n = m["mask"]["size"] if m.get("mask") else 1 << 30
                seen = sum(min(pos + 1, n) for ctx in contexts for pos in range(ctx - new_per_request, ctx))
                keys_read = sum(min(ctx, n + new_per_request - 1) for ctx in contexts)
                add("latent_attention", 2.0 * m["heads"] * seen * (dk + m["kv_rank"]),
                    2 * (keys_read * dk + 2 * tokens * m["heads"] * m["kv_rank"]))
                if m.get("kv_from") is None:
                    add("latent_prepare", 0, tokens * (4 * dk + 2 * dk))
            if f and f["kind"] == "moe":
                top, ff, experts = f["router"]["top"], f["expert"]["ff"], f["router"]["experts"]
                used = min(experts, tokens * top)
                sff = (f.get("shared") or {}).get("ff", 0)          # the shared expert runs inside the same call
                add("routed_experts", 2.0 * tokens * 3 * (top * ff + sff) * width,
                    2 * (used * ff + sff) * 3 * width + tokens * width * (2 + 4))
                add("route_corrected", 2.0 * tokens * experts * width, tokens * width * 2 + experts * width * 4)
    elif cfg.get("architecture") == "Sezanex":
        width = cfg["width"]
        loop = cfg.get("loop")
        runs = [1 + ((loop["times"] - 1) if loop and loop["start"] <= i < loop["stop"] else 0) for i in range(len(cfg["layers"]))]
        for layer, times in zip(cfg["layers"], runs):
            m, f = layer["mixer"], layer["mlp"]
            for _ in range(times):
                # per sub-layer: the stream in and out, the sub-layer's output in, h out
                add("add_dyntanh", 0, (2 if f else 1) * tokens * width * (4 + 4 + 3 + 2))
                if layer["type"] == "mamba2":
                    H, P, N, G = m["heads"], m["vdim"], m["state"], m["groups"]
                    inner, GN = H * P, G * N
                    # per token and head: the state's decay and update (3 N P) and its read (2 N P), however it is cut;
                    # z, x, B, C, dt in, the gated and normed output out, the state in and out
                    add("state_space", 5.0 * tokens * H * N * P,
                        tokens * ((2 * inner + 2 * GN + H) * 2 + inner * 2) + 2 * len(contexts) * H * N * P * 4)
                    # the walk token by token keeps the state float32 on the float32 pipe: two multiply-adds an element
                    work["state_space"]["fp32_flops"] = work["state_space"].get("fp32_flops", 0.0) + 4.0 * tokens * H * N * P
                else:
                    H, G, D, V = m["heads"], m["kv_heads"], m["dim"], m["vdim"]
                    n = m["mask"]["size"] if m.get("mask") else 1 << 30
                    seen = [min(pos + 1, n) for ctx in contexts for pos in range(ctx - new_per_request, ctx)]
                    keys_read = sum(min(ctx, n + new_per_request - 1) for ctx in contexts)
                    add("sink_attention", 2.0 * H * sum(seen) * (D + V), 2 * (keys_read * G * (D + V) + tokens * H * (D + V)))
                    add("qk_norm_rope_write", 0, tokens * ((H + G) * D * 2 * 2 + G * (D + V) * 2 + G * V * 2))
                if f and f["kind"] == "moe":
                    top, ff, experts = f["router"]["top"], f["expert"]["ff"], f["router"]["experts"]
                    used = min(experts, tokens * top)
                    add("input_weighted_experts", 2.0 * tokens * 3 * top * ff * width,
                        2 * used * ff * 3 * width + tokens * width * (2 + 4))
                    add("route_top", 2.0 * tokens * experts * width, tokens * width * 2 + experts * width * 4)
    else:
        width, heads, kv, hd = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
        for _ in range(cfg["num_hidden_layers"]):
            pairs = sum(n * new_per_request - new_per_request * (new_per_request - 1) / 2 for n in contexts)
            add("paged_attention", 2 * heads * pairs * 2 * hd, 2 * (sum(contexts) * 2 * kv * hd + 2 * tokens * heads * hd))
            add("add_rmsnorm", 0, 2 * tokens * width * (4 + 4 + 2 + 2) / 2 * 1.0)
            add("rope_kv_write", 0, tokens * (heads + 2 * kv) * hd * 2 * 2)
            inter = cfg["intermediate_size"]
            add("linear_swiglu", 2 * tokens * 2 * inter * width, 2 * 2 * inter * width + tokens * (width + inter) * 2)
    return work


def _step_kernel_times(engine, family: str, entries_fn, reps: int = 3) -> Dict[str, float]:
    """Microseconds per step and kernel name, eager steps, the best of `reps`."""
    best: Dict[str, float] = {}
    with KernelTimer(engine.kernels, _TIMED[family]) as timer:
        for _ in range(reps + 1):
            entries, finish = entries_fn()
            KernelTimer.hold()
            engine.step(entries)
            got = timer.totals()
            for rid in finish:
                engine.finish(rid)
            for name, us in got.items():
                best[name] = min(best.get(name, float("inf")), us)
    return best


def run_design_comparison(name: str = "bozavik-a", *, prefill_tokens: int = PREFILL_TOKENS, batch: int = 8,
                          context: int = 4096, steps: int = 32, warmup: int = 4, device: str = "cuda:0") -> dict:
    """Prefill and decode throughput of a named model of another design (Bozavik, Pedazen, Sezanex, Bufolorn; random weights) and of the
    dense decoder closest to it at equal size, and, kernel by kernel, how far the design's own kernels are from their
    rooflines beside the like kernels of the dense model (eager steps, CUDA events around each kernel-table call)."""
    from ..engine.step import StepEntry
    from .common import closest_llama

    pk = peaks()
    out = {"model": name, "peaks": pk["source"], "prefill_tokens": prefill_tokens, "decode": {"batch": batch, "context": context}}
    design = RANDOM_MODELS[name].get("architecture")
    if design not in _TIMED:
        raise SystemExit(f"{name!r} is no model of another design; known: "
                         f"{sorted(n for n, c in RANDOM_MODELS.items() if c.get('architecture') in _TIMED)}")
    out["design"] = design
    configs = {design: dict(RANDOM_MODELS[name])}
    configs["Llama"] = closest_llama(configs[design])
    for family, cfg in configs.items():
        vocab = cfg.get("vocab", cfg.get("vocab_size"))
        prompts = Prompts(vocab)
        res = {}
        engine = make_engine(cfg, max_batch=batch, context=context, device=device)
        ids = prompts(prefill_tokens)

        def once():
            engine.step([StepEntry("p", ids, [prefill_tokens - 1])])
            engine.finish("p")

        for _ in range(3):
            once()
        ms = statistics.median(timed(once, 3) for _ in range(3))
        res["prefill_ms"] = round(ms, 3)
        res["prefill_tokens_per_s"] = round(prefill_tokens / ms * 1e3, 1)
        start = context - steps - warmup - 1
        rids = fill_requests(engine, cfg, batch, start, prompts, "synthetic")
        tokens = engine.decode_steps(rids, [1] * batch, warmup)[-1]
        before = engine.kernels.launches
        ms = timed(lambda: engine.decode_steps(rids, tokens, steps), 1) / steps
        res["decode_ms_per_step"] = round(ms, 4)
        res["decode_tokens_per_s"] = round(batch / ms * 1e3, 1)
        res["decode_launches_per_step"] = (engine.kernels.launches - before) // steps
        for rid in rids:
            engine.finish(rid)
        engine.close()
        # kernel by kernel, eagerly
        engine = make_engine(cfg, max_batch=batch, context=context, device=device, cuda_graph=False)
        table = {}
        times = _step_kernel_times(engine, family, lambda: ([StepEntry("p", ids, [prefill_tokens - 1])], ["p"]))
        work = _kernel_work(cfg, prefill_tokens, [prefill_tokens], prefill_tokens)
        table["prefill"] = _roofline_rows(times, work, pk)
        rids = fill_requests(engine, cfg, batch, start, prompts, "synthetic")
        times = _step_kernel_times(engine, family, lambda: ([StepEntry(r, [1], [0]) for r in rids], []))
        held = [engine.cache.length(r) for r in rids]
        work = _kernel_work(cfg, batch, held, 1)
        table["decode"] = _roofline_rows(times, work, pk)
        for rid in rids:
            engine.finish(rid)
        engine.close()
        res["kernels"] = table
        out[family] = res
        del engine
        torch.cuda.empty_cache()
    return out


def _roofline_rows(times: Dict[str, float], work: Dict[str, dict], pk: dict) -> Dict[str, dict]:
    rows = {}
    for name, us in sorted(times.items()):
        name = name.lstrip("_")
        row = {"us": round(us, 1)}
        w = work.get(name)
        if w and us > 0:
            t_flops = w["flops"] / (pk["bf16_tflops"] * 1e12) * 1e6
            t_bytes = w["bytes"] / (pk["hbm_gbs"] * 1e9) * 1e6
            row["roofline_us"] = round(max(t_flops, t_bytes), 2)
            row["bound"] = "tensor" if t_flops > t_bytes else "hbm"
            row["frac"] = round(max(t_flops, t_bytes) / us, 4)
            if w.get("fp32_flops"):
                row["fp32_pipe_us"] = round(w["fp32_flops"] / (fp32_pipe_tflops() * 1e12) * 1e6, 2)
                row["fp32_pipe_frac"] = round(row["fp32_pipe_us"] / us, 4)
        rows[name] = row
    return rows
