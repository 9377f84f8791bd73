"""Serving probes (the roles of the reference's code/ops/stall_probe.py and code/ops/apc_probe.py), run through the
engine's public step API:

  stall   an incumbent request decodes; after ``join_after`` of its steps a newcomer with a long prompt arrives.
          Reported per mixed-prefill cap: the incumbent's inter-token times (median, max = the stall the newcomer's
          prefill causes), the newcomer's time to first token, and how many steps carried prefill beside decode.
          The cap trades the newcomer's wait against the incumbent's stall (``EngineConfig.mixed_prefill_chunk``).
  apc     prefix-cache reuse across turns: turn 1 is generated, then turn 2 = turn 1 + its answer + a follow-up.
          Reported: tokens served from the cache, and turn 2's time to first token against a cold prompt of the same
          length (its first token changed, so nothing matches).

    python -m glm53.utils.serve_probe stall --model full --caps 0 2048 --newcomer-len 32768
    python -m glm53.utils.serve_probe apc --model full --len 8192 --follow-up 256
"""

from __future__ import annotations

import argparse
import json
import time

from ..engine.llm import SamplingParams, State


def _sync():
    import torch
    if torch.cuda.is_available():
        torch.cuda.synchronize()


def _timed_step(engine) -> float:
    t0 = time.perf_counter()
    engine.step()
    _sync()
    return time.perf_counter() - t0


def _req(engine, rid):
    return next((r for r in engine.running if r.rid == rid), None)


def stall(engine, incumbent: list[int], newcomer: list[int], gen: int = 64, join_after: int = 4) -> dict:
    """One incumbent, one newcomer; the engine's current ``mixed_prefill_chunk`` applies."""
    a = engine.add_request(incumbent, SamplingParams(max_tokens=gen, ignore_eos=True))
    while (_req(engine, a) is None or _req(engine, a).state != State.RUNNING) and a not in engine.done:
        engine.step()
    itl, prefill_steps, b, t_join, ttft = [], 0, None, 0.0, None
    n_prev = len((_req(engine, a) or engine.done[a]).output)
    steps = 0
    while a not in engine.done:
        if steps == join_after and b is None:
            b = engine.add_request(newcomer, SamplingParams(max_tokens=1, ignore_eos=True))
            t_join = time.perf_counter()
        prefilling = b is not None and ttft is None
        dt = _timed_step(engine)
        steps += 1
        ra = _req(engine, a) or engine.done.get(a)
        if len(ra.output) > n_prev:
            itl.append(dt * 1e3)                      # time between the incumbent's emissions
            n_prev = len(ra.output)
        if prefilling:
            prefill_steps += 1
            rb = _req(engine, b) or engine.done.get(b)
            if rb is not None and rb.output:
                ttft = (time.perf_counter() - t_join) * 1e3
    while b is not None and b not in engine.done:
        engine.step()
        rb = _req(engine, b) or engine.done.get(b)
        if ttft is None and rb is not None and rb.output:
            ttft = (time.perf_counter() - t_join) * 1e3
    srt = sorted(itl)
    return {"incumbent_steps": len(itl), "itl_median_ms": srt[len(srt) // 2] if srt else None,
            "itl_max_ms": srt[-1] if srt else None, "newcomer_ttft_ms": ttft, "prefill_steps": prefill_steps}


def _ttft(engine, prompt: list[int]) -> tuple[float, int]:
    m0 = engine.metrics["prefix_cached_tokens"]
    t0 = time.perf_counter()
    rid = engine.add_request(prompt, SamplingParams(max_tokens=1, ignore_eos=True))
    while rid not in engine.done:
        engine.step()
    _sync()
    return (time.perf_counter() - t0) * 1e3, engine.metrics["prefix_cached_tokens"] - m0


def apc(engine, prompt: list[int], follow_up: list[int], gen: int = 32) -> dict:
    answer = engine.generate([prompt], SamplingParams(max_tokens=gen, ignore_eos=True))[0]
    turn2 = prompt + answer + follow_up
    warm_ms, cached = _ttft(engine, turn2)
    cold = [turn2[0] ^ 1] + turn2[1:]
    cold_ms, cold_cached = _ttft(engine, cold)
    return {"turn2_tokens": len(turn2), "cached_tokens": cached, "cached_fraction": cached / len(turn2),
            "ttft_warm_ms": warm_ms, "ttft_cold_ms": cold_ms, "cold_cached_tokens": cold_cached}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["stall", "apc"])
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--caps", type=int, nargs="+", default=[0, 2048], help="mixed prefill caps (stall)")
    ap.add_argument("--incumbent-len", type=int, default=1024)
    ap.add_argument("--newcomer-len", type=int, default=8192)
    ap.add_argument("--gen", type=int, default=48)
    ap.add_argument("--len", type=int, default=4096, help="turn-1 prompt length (apc)")
    ap.add_argument("--follow-up", type=int, default=128)
    ap.add_argument("--prefill-chunk", type=int, default=8192)
    args = ap.parse_args(argv)
    import torch
    from ..api.offline import LLM, LLMOptions
    g = torch.Generator().manual_seed(0)
    rnd = lambda n: torch.randint(16, 4096, (n,), generator=g).tolist()
    need = max(args.newcomer_len, args.len + args.gen + args.follow_up) + 256
    llm = LLM(LLMOptions(model=args.model, max_seqs=2, max_model_len=need, prefill_chunk=args.prefill_chunk,
                         checkpoints=4 if args.mode == "apc" else 0))
    if args.mode == "stall":
        inc, new = rnd(args.incumbent_len), rnd(args.newcomer_len)
        res = {"mode": "stall", "runs": []}
        for cap in args.caps:
            llm.engine.cfg.mixed_prefill_chunk = cap
            res["runs"].append({"mixed_prefill_chunk": cap, **stall(llm.engine, inc, new, args.gen)})
    else:
        res = {"mode": "apc", **apc(llm.engine, rnd(args.len), rnd(args.follow_up), args.gen)}
    print(json.dumps(res))
    return res


if __name__ == "__main__":
    main()
