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

PUBLISHED_DECODE_TOK_S = 99.44        # 2x GB10, TP=2, structured workload (accept 7.0/step)
PUBLISHED_PREFILL_TOK_S = 3046.0      # cold 32k prefill
METRIC = "bs1 decode ms/step & tok/s (K=7); 32k cold-prefill tok/s; at 1/2/4/8 B200"

REFERENCE_UNAVAILABLE = ("the reference is a vLLM plugin/overlay kit for an arm64 GB10 (sm_121a) image pulled from "
                         "GHCR; /root/reference has no installable package at its root and its fork package builds "
                         "only sm_121a extensions against an unpublished vLLM build, so it cannot run on B200 here")


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [l.strip().split(", ") for l in self.file.read().splitlines() if l.strip()]
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
    return ap.parse_args()


def main():
    args = parse()
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "metric": METRIC, "unavailable": REFERENCE_UNAVAILABLE}))
        return
    import torch
    import glm53
    from glm53.models import weights as W
    from glm53.models.runtime import Graphed, Runtime, RuntimeConfig
    from glm53.models.session import Sequence
    from glm53.ops.sampling import GreedySampler
    from glm53.parallel import dist as D

    rank, local, world = D.init()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    comm = D.NcclComm() if world > 1 else None
    dev = torch.device("cuda", local)
    cfg = glm53.full_config(args.layers) if args.model == "full" else glm53.tiny_config()
    t0 = time.time()
    w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev)
    torch.cuda.synchronize()
    t_load = time.time() - t0
    K = args.k
    rows = K + 1
    chunk = min(args.prefill_chunk, max(args.context, 16))
    bs = 64
    ctx_cap = args.context + rows * (args.steps + args.warmup + 4) + 64
    if not args.no_prefill:
        ctx_cap = max(ctx_cap, args.prefill_tokens + 64)
    max_blocks = (ctx_cap + bs - 1) // bs
    rc = RuntimeConfig(max_rows=max(chunk, 16), max_seqs=1, kv_slots=max_blocks * bs, block_size=bs,
                       max_blocks=max_blocks, decode_rows=16, mla_splits=4, logit_rows=16)
    rt = Runtime(w, rc, comm=comm)
    seq = Sequence(rt)
    sampler = GreedySampler(16, world, w.rank * w.head.n, comm, dev)
    gen = torch.Generator().manual_seed(1234)
    stream = torch.cuda.current_stream()

    def barrier_sync():
        if comm:
            comm.barrier()
        torch.cuda.synchronize()

    # ---------------- cold prefill (separate sequence state: reset afterwards) ----------------
    prefill = None
    if not args.no_prefill:
        ptoks = torch.randint(0, cfg.vocab, (args.prefill_tokens,), generator=gen).tolist()
        seq.prefill(ptoks[:min(2048, len(ptoks))], chunk=min(chunk, 2048))      # warm-up (kernels, allocator)
        seq.reset()
        barrier_sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        seq.prefill(ptoks, chunk=chunk)
        e1.record(stream)
        barrier_sync()
        ms = e0.elapsed_time(e1)
        ms = comm.max_scalar(ms) if comm else ms
        prefill = {"tokens": args.prefill_tokens, "chunk": chunk, "ttft_s": ms / 1e3,
                   "tok_s": args.prefill_tokens / (ms / 1e3), "vs_published": args.prefill_tokens / (ms / 1e3) /
                   PUBLISHED_PREFILL_TOK_S}
        seq.reset()

    # ---------------- context for decode ----------------
    ctx = torch.randint(0, cfg.vocab, (args.context,), generator=gen).tolist()
    logits = seq.prefill(ctx, chunk=chunk)
    last = int(sampler(logits)[0].item())

    # pinned staging of each step's inputs and outputs (the end-to-end path's H2D / D2H)
    h_in = torch.zeros(rows, dtype=torch.int32, pin_memory=True)
    h_out = torch.zeros(rows, dtype=torch.int32, pin_memory=True)

    def stage_window(tokens):
        seq.stage(tokens, list(range(rows)))
        seq._window = rows

    stage_window([last] + [0] * K)
    fwd = (lambda: rt.forward(rows, keep_window=True))
    if not args.no_graph:
        g_fwd = Graphed(fwd)
        rt.stage_commit([seq._seq_desc(rows)])
        g_commit = Graphed(lambda: rt.commit(None, replay=False))
    drafts = torch.randint(0, cfg.vocab, (args.steps + args.warmup + 2, K), generator=gen)

    def step(i, tok):
        h_in[0] = tok
        h_in[1:] = drafts[i]
        stage_window(h_in.tolist())
        lg = g_fwd() if not args.no_graph else fwd()
        tgt = sampler(lg)                                  # greedy target tokens of every row
        h_out.copy_(tgt, non_blocking=True)                # D2H of the step result
        if args.no_graph:
            rt.commit([seq._seq_desc(rows)], replay=False)
        else:
            rt.stage_commit([seq._seq_desc(rows)])      # the commit graph reads the staged descriptor
            g_commit()
        seq.cur = 1 - seq.cur
        seq.pos += rows
        return tgt

    for i in range(args.warmup):
        step(i, last)
        torch.cuda.synchronize()
        last = int(h_out[-1])
    barrier_sync()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    wall0 = time.perf_counter()
    for i in range(args.steps):
        step(args.warmup + i, last)
        torch.cuda.synchronize()                            # the host reads the emitted tokens every step
        last = int(h_out[-1])
    e1.record(stream)
    barrier_sync()
    wall = time.perf_counter() - wall0
    ck = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms = comm.max_scalar(ms) if comm else ms
    wall = comm.max_scalar(wall) if comm else wall
    ms_step = ms / args.steps
    tok_s = rows / (ms_step / 1e3)

    # kernel launches of one step (counted with the profiler on an untimed step)
    launches = None
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step(args.warmup + args.steps, last)
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
        ours = [n for n in names if "g53" in n]
        launches = {"per_step_ours": len(ours), "per_step_total": len(names)}
    except Exception as e:  # pragma: no cover
        launches = {"error": str(e)[:200]}

    if rank == 0:
        out = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": tok_s / PUBLISHED_DECODE_TOK_S, "dtype": "bf16 activations / fp8 e4m3 dense / EXL3 4bpw",
            "data": "synthetic: random-init weights (seed 0), uniform random token ids",
            "config": {"model": f"glm-5.3-flash {cfg.layers} layers, 288 experts top-8, EXL3 4bpw, vocab {cfg.vocab}"
                       if args.model == "full" else "glm53-tiny", "global_batch": 1, "seq_len": args.context,
                       "parallelism": f"tp{world}", "K": K, "tokens_per_step": rows,
                       "acceptance": "forced (all K drafts accepted)", "cuda_graph": not args.no_graph,
                       "l2": "inputs larger than L2: each step streams tens of GB of weights"},
            "prefill": prefill,
            "e2e": {"value": rows * args.steps / wall, "unit": "tok/s",
                    "h2d_bytes_per_step": int(h_in.numel() * 4), "d2h_bytes_per_step": int(h_out.numel() * 4),
                    "note": "host loop: pinned H2D of the window tokens, graph replay, D2H of the verified tokens"},
            "gpu_launches": (launches.get("per_step_ours", 0) * args.steps) if isinstance(launches, dict) else None,
            "launch_detail": launches,
            "clocks": ck,
            "load_s": t_load,
        }
        print(json.dumps(out))
    if not args.no_graph:
        del g_fwd, g_commit
    if comm:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
