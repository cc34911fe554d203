"""bench.py --gpus 1 --steps K --warmup W: decode and prefill throughput of the engine.

The model has the layer sizes of Llama 3.2 1B with random weights. The headline `value` is
decoded tokens per second at batch 8 with every request holding about `context` tokens; a
"step" is one decode step. It prints ONE JSON line. The engine runs on one GPU: for
--gpus N > 1 it prints one line that says so and exits with 2. The measuring code is the
package's (tt_transformers_b200.cli.measure), shared with bin/benchmark.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FULL_LAYERS = 16
POINT_STEPS = 64          # the other batch sizes are timed over at least this many steps, whatever --steps says


def reference_arm() -> dict:
    """The reference's own generation path needs its vendor's accelerator library (ttnn) and a
    Tenstorrent device. If the package under baseline/_ref and that library import, its stock
    loader would be driven here; where they do not, the arm says so in one line."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "tt_transformers")):
        return {"impl": "reference", "unavailable": "baseline/_ref holds no installed tt_transformers package"}
    sys.path.insert(0, ref)
    try:
        import ttnn  # noqa: F401
    except Exception as e:            # not installed here: there is no wheel of it offline and no CUDA backend
        return {"impl": "reference", "unavailable":
                f"tt_transformers is installed under baseline/_ref (--no-deps), but its accelerator library "
                f"cannot be imported ({type(e).__name__}: {e}); every forward op of the reference is a call into it"}
    return {"impl": "reference", "unavailable": "ttnn imported, but no Tenstorrent device is present on a B200 box"}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=64)
    parser.add_argument("--warmup", type=int, default=8)
    parser.add_argument("--impl", default="ours", choices=("ours", "reference"))
    parser.add_argument("--batch", type=int, default=8)
    parser.add_argument("--context", type=int, default=8192)
    parser.add_argument("--layers", type=int, default=FULL_LAYERS)
    parser.add_argument("--points", default="1,64", help="other decode batch sizes to report, comma separated")
    parser.add_argument("--skip-prefill", action="store_true", help="leave the prefill measurement out (for profiling decode)")
    parser.add_argument("--skip-e2e", action="store_true", help="leave the end-to-end measurement out (for profiling)")
    parser.add_argument("--design", default=None,
                        help="instead of the default workload: prefill and decode throughput of a named random model of "
                             "another design (bozavik-a, bozavik-b, pedazen-a, pedazen-b, sezanex-a, sezanex-b, bufolorn-a, bufolorn-b) beside the closest dense model at equal size, with "
                             "the design's own kernels against their rooflines")
    parser.add_argument("--fill", default="prefill", choices=("prefill", "synthetic"),
                        help="how the cache gets its context before decoding: through the engine's own prefill, "
                             "or filled with random numbers (faster; decode time does not depend on the values)")
    args = parser.parse_args(argv)

    if args.impl == "reference":
        print(json.dumps(reference_arm()))
        return 0
    if args.gpus != 1:
        print(f"bench.py: this engine runs on one GPU; --gpus {args.gpus} is not supported")
        return 2
    warmup = max(args.warmup, 3)

    if args.design:
        from tt_transformers_b200.cli import measure

        context = min(args.context, 4096)
        result = measure.run_design_comparison(args.design, batch=args.batch, context=context,
                                               steps=min(args.steps, 32), warmup=warmup)
        own = result[result["design"]]
        print(json.dumps({"metric": f"decode tokens/s, {args.design} sizes, batch {args.batch}", "value": own["decode_tokens_per_s"],
                          "unit": "tokens/s", "n_gpus": 1, "steps": min(args.steps, 32), "warmup": warmup,
                          "ms_per_step": own["decode_ms_per_step"], "higher_is_better": True, "dtype": "bf16",
                          "data": "synthetic: random weights, uniform-random token ids",
                          "config": {"model": args.design, "global_batch": args.batch, "seq_len": context}, "comparison": result}))
        return 0

    from tt_transformers_b200.cli import measure
    from tt_transformers_b200.engine.llm import LLM

    sampler = measure.ClockSampler()      # runs for the whole measurement; each timed region takes its own samples
    cfg = dict(measure.model_config("1b"), num_hidden_layers=args.layers)
    pk = measure.peaks()
    point_batches = [int(x) for x in args.points.split(",") if x]
    max_batch = max([args.batch] + point_batches)
    engine = measure.make_engine(cfg, max_batch=max_batch, context=args.context)
    llm = LLM(engine)
    prompts = measure.Prompts(cfg["vocab_size"])

    prefill = {"value": None, "tokens": measure.PREFILL_TOKENS, "ms": None, "frac": None}
    ttft = None
    if not args.skip_prefill:
        prefill = measure.measure_prefill(engine, cfg, args.layers, pk, prompts=prompts)
        ttft = measure.measure_ttft(engine, cfg, 128, prompts=prompts)

    head = measure.measure_decode(engine, cfg, args.layers, pk, args.batch, args.context, args.steps, warmup,
                                  sampler=sampler, how=args.fill, prompts=prompts)
    points, points_ms = {}, {}
    for b in point_batches:
        p = measure.measure_decode(engine, cfg, args.layers, pk, b, args.context, max(POINT_STEPS, args.steps), warmup,
                                   how=args.fill, prompts=prompts)
        points[f"decode_b{b}"] = p["tokens_per_s"]
        points_ms[f"decode_b{b}"] = {"ms_per_step": p["ms_per_step"], "steps": p["steps"], "frac": p["roofline"]["frac"]}

    e2e = None
    if not args.skip_e2e:
        e2e = measure.measure_e2e(llm, cfg, args.batch, args.context, args.steps, warmup, prompts=prompts, how=args.fill)
        e2e.pop("ms_per_step", None)

    line = {
        "metric": "decode tokens/s, Llama 3.2 1B sizes, batch 8", "value": head["tokens_per_s"], "unit": "tokens/s",
        "n_gpus": 1, "steps": args.steps, "warmup": warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random weights N(0, 0.02), uniform-random token ids",
        "config": {"model": "llama-3.2-1b-sizes", "layers": args.layers, "layers_full": FULL_LAYERS,
                   "hidden": cfg["hidden_size"], "heads": cfg["num_attention_heads"],
                   "kv_heads": cfg["num_key_value_heads"], "head_dim": cfg["head_dim"],
                   "intermediate": cfg["intermediate_size"], "vocab": cfg["vocab_size"], "global_batch": args.batch,
                   "seq_len": args.context, "page_size": measure.PAGE, "prefill_tokens": measure.PREFILL_TOKENS,
                   "parallelism": "single-gpu", "cache_fill": args.fill,
                   "l2": "inputs larger than L2 (weights and cache are re-read every step)",
                   "peaks": pk["source"]},
        "clocks": head["clocks"], "e2e": e2e, "gpu_launches": head["gpu_launches"], "prefill": prefill,
        "roofline": {k: head["roofline"][k] for k in ("bound", "achieved", "peak", "unit", "frac")},
        "points": points, "points_ms": points_ms, "ttft": ttft,
    }
    sampler.stop()
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
