"""Sampled-decoding bench (the role of the reference's code/kit/tools/bench_sampled.py:1-30): temperature sampling
with fixed seeds, one request at a time through the engine, and per request the speculative statistics that the
greedy / forced-acceptance headline bench cannot show:

  accepted tokens / step   1 + accepted drafts / verify windows
  per-position acceptance  windows whose draft at position i was accepted / windows
  draft tokens / step      drafted tokens / windows (the adaptive K actually verified)
  tok/s, ms/step           generated tokens and decode wall time over the request's decode steps

Request i uses seed = seed_base + i, so two runs (e.g. standard against block verification, or two builds) draw
the same seeds; `--compare A.json B.json` prints the per-metric means side by side.

    python -m glm53.utils.bench_sampled --model full --out standard.json --seeds 4 --max-tokens 256
    python -m glm53.utils.bench_sampled --model full --block-verify --out block.json
    python -m glm53.utils.bench_sampled --compare standard.json block.json
"""

from __future__ import annotations

import argparse
import json
import time


def window_stats(m0: dict, m1: dict, tokens: int, seconds: float) -> dict:
    """Statistics of the decode steps between two snapshots of the engine metrics."""
    windows = m1["spec_windows"] - m0["spec_windows"]
    steps = m1["steps"] - m0["steps"]
    out = {"windows": windows, "steps": steps, "tokens": tokens,
           "tok_s": tokens / seconds if seconds > 0 else None,
           "ms_per_step": seconds * 1e3 / steps if steps else None}
    if windows:
        acc = m1["spec_accepted"] - m0["spec_accepted"]
        out["accepted_per_step"] = 1.0 + acc / windows
        out["draft_tokens_per_step"] = (m1["spec_drafts"] - m0["spec_drafts"]) / windows
        pp0, pp1 = m0["spec_accepted_per_pos"], m1["spec_accepted_per_pos"]
        out["acceptance_per_position"] = [(b - a) / windows for a, b in zip(pp0, pp1)][:8]
    return out


def snapshot(metrics: dict) -> dict:
    return {k: (list(v) if isinstance(v, list) else v) for k, v in metrics.items()}


def run(engine, prompts: list[list[int]], params_for) -> list[dict]:
    """One request at a time: prefill it, then time its decode steps."""
    from ..engine.llm import State
    res = []
    for i, prompt in enumerate(prompts):
        rid = engine.add_request(prompt, params_for(i))
        while not any(r.rid == rid and r.state == State.RUNNING for r in engine.running):
            if rid in engine.done:
                break
            engine.step()
        r0 = next((r for r in engine.running if r.rid == rid), None)
        n0 = len(r0.output) if r0 else 0
        m0 = snapshot(engine.metrics)
        t0 = time.perf_counter()
        while rid not in engine.done:
            engine.step()
        dt = time.perf_counter() - t0
        out = engine.done[rid].output
        res.append({"seed_index": i, **window_stats(m0, engine.metrics, len(out) - n0, dt)})
    return res


def summary(rows: list[dict]) -> dict:
    keys = ("accepted_per_step", "draft_tokens_per_step", "tok_s", "ms_per_step")
    out = {}
    for k in keys:
        vals = [r[k] for r in rows if r.get(k) is not None]
        out[k] = sum(vals) / len(vals) if vals else None
    pos = [r["acceptance_per_position"] for r in rows if "acceptance_per_position" in r]
    if pos:
        out["acceptance_per_position"] = [sum(p[i] for p in pos) / len(pos) for i in range(len(pos[0]))]
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="full")
    ap.add_argument("--seeds", type=int, default=4)
    ap.add_argument("--seed-base", type=int, default=1000)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--temperature", type=float, default=1.0)
    ap.add_argument("--top-p", type=float, default=0.95)
    ap.add_argument("--block-verify", action="store_true")
    ap.add_argument("--out", default="")
    ap.add_argument("--compare", nargs=2, default=None)
    args = ap.parse_args(argv)
    if args.compare:
        a, b = (json.load(open(p)) for p in args.compare)
        res = {"a": args.compare[0], "b": args.compare[1], "summary_a": a["summary"], "summary_b": b["summary"]}
        print(json.dumps(res))
        return res
    import torch
    from ..api.offline import LLM, LLMOptions
    from ..engine.llm import SamplingParams
    llm = LLM(LLMOptions(model=args.model, max_seqs=1, max_model_len=args.prompt_len + args.max_tokens + 64,
                         prefill_chunk=min(8192, args.prompt_len), speculative=True, checkpoints=0,
                         block_verify=args.block_verify))
    g = torch.Generator().manual_seed(args.seed_base)
    prompts = [torch.randint(16, llm.cfg.vocab, (args.prompt_len,), generator=g).tolist()
               for _ in range(args.seeds)]
    params = lambda i: SamplingParams(max_tokens=args.max_tokens, temperature=args.temperature, top_p=args.top_p,
                                      seed=args.seed_base + i, ignore_eos=True)
    rows = run(llm.engine, prompts, params)
    res = {"mode": "block" if args.block_verify else "standard", "temperature": args.temperature,
           "top_p": args.top_p, "requests": rows, "summary": summary(rows)}
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f)
    print(json.dumps(res["summary"]))
    return res


if __name__ == "__main__":
    main()
