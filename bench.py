#!/usr/bin/env python
"""Headline benchmark of the reference: single-stream speculative decode with K=7 drafts and
forced acceptance (ms/step, tok/s) on the full GLM-5.3-Flash architecture, plus cold prefill tok/s.

Model: 45 layers (34 KDA + 11 MLA/DSA), hidden 4096, 288 EXL3 4-bpw experts top-8 + shared, 4 mHC streams,
vocab 154,880, fp8 e4m3 MLA latent cache; random-init weights (seed 0) and uniform random token ids (no network).
Each decode step: a verify window of K+1 rows through the target (one CUDA graph), the greedy verifier, the commit,
and a draft of K tokens by the block drafter; K+1 tokens are emitted per step (acceptance forced to K).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--context 4096] [--k 7] [--prefill-tokens 32768]
  python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...     (tensor parallel over N GPUs)
  python bench.py --impl reference ...      (the reference's own stack; prints its "unavailable" line here)

Timing: W untimed steps, then K steps bracketed by barrier + synchronize, CUDA events on the launching stream, max
over ranks.  Every step streams ~30 GB of expert and dense weights (>> the 126 MB L2), so no L2 flush is needed.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PUBLISHED_DECODE_TOK_S = 99.44        # the reference's published figure: 2x GB10, TP=2, structured workload (accept 7.0/step)
PUBLISHED_PREFILL_TOK_S = 3046.0      # the reference's published figure: cold 32k prefill
METRIC = "bs1 decode ms/step & tok/s (K=7); 32k cold-prefill tok/s; at 1/2/4/8 B200"

REFERENCE_UNAVAILABLE = ("the reference is a vLLM plugin/overlay kit for an arm64 GB10 (sm_121a) image pulled from "
                         "GHCR; the reference repository has no installable package at its root and its fork package builds "
                         "only sm_121a extensions against an unpublished vLLM build, so it cannot run on B200 here")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms; only the samples taken between mark() and stop()
    (the timed region) are reported (at least the first sample after mark(), for very short regions)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None
        self.n0 = 0

    def _lines(self) -> list[str]:
        self.file.flush()
        with open(self.file.name) as f:
            return [l.strip() for l in f.read().splitlines() if l.strip()]

    def start(self):
        """Start sampling and wait (at most 3 s) until the first sample is written."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "50"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 3.0 and not self._lines():
            time.sleep(0.02)

    def mark(self):
        """The timed region starts now."""
        if self.proc is not None:
            self.n0 = len(self._lines())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t0 = time.time()
        while time.time() - t0 < 1.0 and len(self._lines()) <= self.n0:
            time.sleep(0.01)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [l.split(", ") for l in self._lines()[self.n0:]]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--k", type=int, default=7)
    ap.add_argument("--prefill-tokens", type=int, default=32768)
    ap.add_argument("--prefill-chunk", type=int, default=8192)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--layers", type=int, default=45)
    ap.add_argument("--model", default="full", choices=["full", "tiny"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--ep", action="store_true", help="routed experts expert-parallel over the GPUs (TP elsewhere)")
    return ap.parse_args()


def main():
    args = parse()
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": REFERENCE_UNAVAILABLE}))
        return
    import torch
    from glm53.api.offline import LLM, LLMOptions
    from glm53.engine.llm import SamplingParams, State
    from glm53.parallel import dist as D

    rank, local, world = D.init()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    comm = D.NcclComm() if world > 1 else None
    K = args.k
    rows = K + 1
    chunk = args.prefill_chunk
    max_len = max(args.context, args.prefill_tokens if not args.no_prefill else 0) + rows * (args.steps +
                                                                                              args.warmup + 8) + 64
    t0 = time.time()
    llm = LLM(LLMOptions(model=args.model, layers=args.layers if args.layers != 45 else None, max_seqs=1,
                         max_model_len=max_len, prefill_chunk=chunk, speculative=True, k_fixed=K,
                         force_accept=True, checkpoints=0, cuda_graphs=not args.no_graph, ep=args.ep), comm=comm,
              rank=rank, world=world)
    torch.cuda.synchronize()
    t_load = time.time() - t0
    eng = llm.engine
    cfg = llm.cfg
    gen = torch.Generator().manual_seed(1234)
    stream = torch.cuda.current_stream()

    def barrier_sync():
        if comm:
            comm.barrier()
        torch.cuda.synchronize()

    def run_until(pred):
        while not pred():
            eng.step()

    # ---------------- cold prefill through the engine: TTFT of a max_tokens=1 request ----------------
    prefill = None
    if not args.no_prefill:
        warm = torch.randint(0, cfg.vocab, (min(chunk, args.prefill_tokens),), generator=gen).tolist()
        rid = eng.add_request(warm, SamplingParams(max_tokens=1, ignore_eos=True))     # warm-up: kernels, allocator
        run_until(lambda: rid in eng.done)
        ptoks = torch.randint(0, cfg.vocab, (args.prefill_tokens,), generator=gen).tolist()
        barrier_sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.perf_counter()
        e0.record(stream)
        rid = eng.add_request(ptoks, SamplingParams(max_tokens=1, ignore_eos=True))
        run_until(lambda: rid in eng.done)
        e1.record(stream)
        barrier_sync()
        wall = time.perf_counter() - w0
        ms = e0.elapsed_time(e1)
        ms = comm.max_scalar(ms) if comm else ms
        wall = comm.max_scalar(wall) if comm else wall
        prefill = {"tokens": args.prefill_tokens, "chunk": chunk, "ttft_s": ms / 1e3,
                   "tok_s": args.prefill_tokens / (ms / 1e3), "e2e_tok_s": args.prefill_tokens / wall,
                   "vs_published": args.prefill_tokens / (ms / 1e3) / PUBLISHED_PREFILL_TOK_S}

    # ---------------- decode: a request with a random context, K drafts per step, acceptance forced ----------------
    ctx = torch.randint(0, cfg.vocab, (args.context,), generator=gen).tolist()
    rid = eng.add_request(ctx, SamplingParams(max_tokens=max_len - args.context - 8, ignore_eos=True))
    run_until(lambda: eng.running and eng.running[0].state == State.RUNNING)
    req = eng.running[0]
    for _ in range(args.warmup):
        eng.step()
    barrier_sync()
    n_tok0 = len(req.output)
    clocks = ClockSampler(local)
    clocks.start()
    barrier_sync()
    clocks.mark()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        eng.step()                       # stage (pinned H2D) -> verify graph -> sample -> D2H tokens -> commit -> draft
    e1.record(stream)
    barrier_sync()
    wall = time.perf_counter() - wall0
    ck = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms = comm.max_scalar(ms) if comm else ms
    wall = comm.max_scalar(wall) if comm else wall
    emitted = len(req.output) - n_tok0
    ms_step = ms / args.steps
    tok_s = emitted / (ms / 1e3)
    h2d = int(getattr(llm.backend.rt.batch, "h2d_bytes", 0))

    launches = None
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            eng.step()
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
        ours = [n for n in names if "g53" in n]
        launches = {"per_step_ours": len(ours), "per_step_total": len(names)}
    except Exception as e:  # pragma: no cover
        launches = {"error": str(e)[:200]}

    # ---------------- correctness check (untimed): greedy tokens with real verification ----------------
    # acceptance is no longer forced: every emitted token is the target's own greedy choice, so the tokens of
    # this check should agree across GPU counts; the smallest top-1 / top-2 log-probability gap says how close a
    # position was to a tie (a divergence between GPU counts at a near-tie is rounding, not a fault)
    eng.abort(rid)
    eng.cfg.force_accept = False
    cprompt = torch.randint(0, cfg.vocab, (256,), generator=torch.Generator().manual_seed(99)).tolist()
    cid = eng.add_request(cprompt, SamplingParams(max_tokens=16, ignore_eos=True, logprobs=5))
    run_until(lambda: cid in eng.done)
    creq = eng.done[cid]
    ctoks = list(creq.output[:16])
    gaps = []
    for lp, top in creq.logprobs[:16]:
        v = sorted(top.values(), reverse=True)
        gaps.append(v[0] - v[1] if len(v) > 1 else float("inf"))
    import hashlib
    first = sorted(creq.logprobs[0][1].items(), key=lambda kv: -kv[1]) if creq.logprobs else []
    check = {"greedy_tokens": ctoks, "sha16": hashlib.sha256(json.dumps(ctoks).encode()).hexdigest()[:16],
             "min_top2_gap": min(gaps) if gaps else None, "top2_gaps": [round(x, 4) for x in gaps],
             "first_top5": [[int(t), round(float(v), 4)] for t, v in first[:5]],
             "prompt": "256 uniform random ids (seed 99)",
             "note": "random-init weights make the greedy sequence sensitive to rounding: at 1 GPU, exact W8A16 "
                     "instead of W8A8 on two prefill projections (GLM53_PREFILL_W8A8=none) already changes the "
                     "first token; across GPU counts compare first_top5 (ids and log-probabilities)"}

    if rank == 0:
        out = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": tok_s / PUBLISHED_DECODE_TOK_S,
            "dtype": "bf16 activations; fp8 e4m3 dense weights; EXL3 4-bpw experts; fp8 latent KV",
            "data": "synthetic: random-init weights (seed 0), uniform random token ids",
            "config": {"model": f"glm-5.3-flash {cfg.layers} layers (34 KDA + 11 MLA/DSA), 288 experts top-8 + shared,"
                                f" EXL3 4bpw, vocab {cfg.vocab}" if args.model == "full" else "glm53-tiny",
                       "global_batch": 1, "seq_len": args.context,
                       "parallelism": f"tp{world}" + (f"+ep{world}" if args.ep and world > 1 else ""), "K": K,
                       "tokens_per_step": rows, "acceptance": "forced (all K drafts accepted)",
                       "drafter": "1-layer block drafter (grouped dynamic conv, CUDA graph) in every step",
                       "cuda_graph": not args.no_graph,
                       "l2": "inputs larger than L2: every step streams ~35 GB of weights (no flush needed)"},
            "prefill": prefill,
            "e2e": {"value": emitted / wall, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": 4 * rows,
                    "note": "public engine API (LLMEngine.step): pinned H2D of the window, D2H of verified tokens"},
            "gpu_launches": (launches.get("per_step_ours", 0) * args.steps) if isinstance(launches, dict) else None,
            "launch_detail": launches,
            "clocks": ck,
            "check": check,
            "load_s": t_load,
        }
        print(json.dumps(out))
    llm.backend._graphs.clear()
    if comm:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
