"""Step-level profiles of the serving path on one GPU.

  python -m glm53.utils.step_profile forward --rows 8        kernel breakdown of one decode window forward (CUDA graph)
  torchrun --nproc-per-node 4 --master-addr 127.0.0.1 -m glm53.utils.step_profile forward --rows 8
                                                              the same per rank of a tensor-parallel group
  python -m glm53.utils.step_profile prefill --chunk 4096    kernel breakdown of one prefill chunk (context = chunk)
  torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m glm53.utils.step_profile prefill --chunk 8192
                                                              the same on rank 0 of a tensor-parallel group
  python -m glm53.utils.step_profile engine --k 7            wall time of each phase of LLMEngine.step()

``forward`` / ``prefill`` aggregate device time per kernel name with torch.profiler (CUDA activity only).
``engine`` runs a speculative decode through the public engine API and times each backend call (with a
synchronize before and after, so device and host time of a phase are attributed to it) next to the plain step time
measured with no instrumentation.  Random-init weights; synthetic token ids.
"""

from __future__ import annotations

import argparse
import collections
import json
import time

import torch


def _kernel_table(fn, reps: int = 1, top: int = 30, marginal: bool = False):
    """Device time per kernel name over ``reps`` calls of ``fn``.  With ``marginal``, each kernel is charged the
    time from the latest end of any earlier kernel to its own end (zero if it ended earlier): the critical-path
    cost of the kernel, which excludes the time a programmatic-dependent kernel spends waiting for its
    predecessor and includes the launch gap before it.  Marginal times add up to the span of the calls."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    evs = [e for e in prof.events() if e.device_type.name == "CUDA"]
    if marginal:
        evs.sort(key=lambda e: (e.time_range.end, e.time_range.start))
        last = None
        for e in evs:
            a = agg[e.name[:100]]
            a[0] += 1
            t0 = e.time_range.start if last is None else max(last, e.time_range.start)
            a[1] += max(0.0, e.time_range.end - t0)
            last = e.time_range.end if last is None else max(last, e.time_range.end)
    else:
        for e in evs:
            a = agg[e.name[:100]]
            a[0] += 1
            a[1] += e.device_time_total
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    total = sum(v[1] for v in agg.values()) / reps
    return total, [(n, c // reps, t / reps) for n, (c, t) in rows[:top]]


def _runtime(cfg, rows: int, ctx: int):
    """Runtime + sequence on this process's GPU; under torchrun (WORLD_SIZE > 1) the weights are this rank's
    tensor-parallel shard and the runtime reduces over NCCL (and the fused peer exchange)."""
    from ..models import weights as W
    from ..models.runtime import Runtime, RuntimeConfig
    from ..models.session import Sequence
    from ..parallel import dist as D
    rank, local, world = D.init()
    comm = D.NcclComm() if world > 1 else None
    dev = torch.device("cuda", local)
    w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, rank=rank, world=world, device=dev)
    bs = 64
    blocks = (ctx + rows * 8 + bs - 1) // bs + 2
    rc = RuntimeConfig(max_rows=max(rows, 16), max_seqs=1, kv_slots=blocks * bs, block_size=bs, max_blocks=blocks)
    rt = Runtime(w, rc, comm=comm)
    return rt, Sequence(rt)


def _rank0() -> bool:
    import torch.distributed as dist
    return not dist.is_initialized() or dist.get_rank() == 0


def cmd_forward(a):
    """One decode window of ``rows`` distinct random tokens (so the routed experts are those of real text, about 57
    distinct of 288 for 8 rows) replayed as a CUDA graph: the window's time, and per kernel both the summed device
    time and the marginal (critical-path) time.  Under torchrun every rank prints its table; compare rank 0 with
    the slowest rank."""
    from .. import full_config
    from ..models.runtime import Graphed
    cfg = full_config()
    rt, seq = _runtime(cfg, max(a.chunk, a.rows), a.context + a.rows * 16)
    g = torch.Generator().manual_seed(0)
    seq.prefill(torch.randint(0, cfg.vocab, (a.context,), generator=g).tolist(), chunk=a.chunk)
    R = a.rows
    toks = torch.randint(0, cfg.vocab, (R,), generator=g).tolist()
    seq.stage(toks, list(range(R)))
    seq._window = R
    graph = Graphed(lambda: rt.forward(R, keep_window=True))
    for _ in range(3):
        graph()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        graph()
    e1.record()
    torch.cuda.synchronize()
    window_us = e0.elapsed_time(e1) * 100.0
    total, rows = _kernel_table(graph, reps=4, top=a.top)
    mtotal, mrows = _kernel_table(graph, reps=4, top=a.top, marginal=True)
    import torch.distributed as dist
    tp = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    spans = [window_us]
    if tp > 1:
        t = torch.tensor([window_us], device=rt.device)
        out = [torch.zeros_like(t) for _ in range(tp)]
        dist.all_gather(out, t)
        spans = [float(x.item()) for x in out]
    lines = [json.dumps({"mode": "forward", "tp": tp, "rank": rank, "rows": R, "context": a.context,
                         "graph_window_us": window_us, "window_us_per_rank": spans,
                         "kernel_sum_us": total, "marginal_sum_us": mtotal})]
    mt = dict((n, t) for n, _, t in mrows)
    lines.append(f"{'marginal':>10} {'device':>10} {'count':>6}  kernel")
    for n, c, t in rows:
        lines.append(f"{mt.get(n, 0.0):8.1f}us {t:8.1f}us {c:6d}x  {n}")
    for r in range(tp):
        if r == rank:
            print("\n".join(lines), flush=True)
        if tp > 1:
            dist.barrier()
    if tp > 1:
        dist.destroy_process_group()


def cmd_prefill(a):
    from .. import full_config
    cfg = full_config()
    CH = a.chunk
    rt, seq = _runtime(cfg, CH, 3 * CH)
    g = torch.Generator().manual_seed(0)
    toks = torch.randint(0, cfg.vocab, (3 * CH,), generator=g).tolist()
    seq.prefill(toks[:CH], chunk=CH)
    total, rows = _kernel_table(lambda: seq.prefill(toks[CH:2 * CH], chunk=CH))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    seq.prefill(toks[2 * CH:], chunk=CH)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    import torch.distributed as dist
    tp = dist.get_world_size() if dist.is_initialized() else 1
    if _rank0():
        print(json.dumps({"mode": "prefill", "tp": tp, "chunk": CH, "kernel_sum_ms": total / 1e3,
                          "timed_chunk_ms": ms, "tok_s": CH / (ms / 1e3)}))
        for n, c, t in rows:
            print(f"{t / 1e3:10.2f} ms {c:6d}x  {n}")
    if tp > 1:
        dist.barrier()
        dist.destroy_process_group()


def cmd_engine(a):
    from ..api.offline import LLM, LLMOptions
    from ..engine.llm import SamplingParams, State
    from ..parallel import dist as D
    K = a.k
    rank, _, world = D.init()
    comm = D.NcclComm() if world > 1 else None
    llm = LLM(LLMOptions(model="full", max_seqs=1, max_model_len=a.context + (K + 1) * (2 * a.steps + 16) + 64,
                         prefill_chunk=4096, speculative=True, k_fixed=K, force_accept=True, checkpoints=0),
              comm=comm, rank=rank, world=world)
    eng = llm.engine
    g = torch.Generator().manual_seed(0)
    ctx = torch.randint(0, llm.cfg.vocab, (a.context,), generator=g).tolist()
    eng.add_request(ctx, SamplingParams(max_tokens=(K + 1) * (2 * a.steps + 8), ignore_eos=True))
    while not (eng.running and eng.running[0].state == State.RUNNING):
        eng.step()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    plain = (time.perf_counter() - t0) * 1e3 / a.steps

    acc = collections.defaultdict(float)

    def wrap(obj, name, label):
        f = getattr(obj, name)

        def timed(*args, **kw):
            torch.cuda.synchronize()
            s = time.perf_counter()
            out = f(*args, **kw)
            torch.cuda.synchronize()
            acc[label] += time.perf_counter() - s
            return out
        setattr(obj, name, timed)

    b = eng.b
    for name in ("verify", "argmax", "commit", "draft", "hidden"):
        wrap(b, name, "backend." + name)
    wrap(eng.kv, "commit_tokens", "kv.commit_tokens")
    wrap(eng, "_emit", "engine._emit")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        eng.step()
    torch.cuda.synchronize()
    inst = (time.perf_counter() - t0) * 1e3 / a.steps
    phases = {k: v * 1e3 / a.steps for k, v in sorted(acc.items(), key=lambda kv: -kv[1])}
    total, rows = _kernel_table(lambda: [eng.step() for _ in range(2)], reps=1, top=a.top)
    mtotal, mrows = _kernel_table(lambda: [eng.step() for _ in range(2)], reps=1, top=a.top, marginal=True)
    mt = dict((n, t) for n, _, t in mrows)
    if rank == 0:
        print(json.dumps({"mode": "engine", "tp": world, "k": K, "context": a.context, "plain_step_ms": plain,
                          "instrumented_step_ms": inst, "phases_ms": phases,
                          "unattributed_ms": inst - sum(phases.values()), "kernel_sum_us_per_step": total / 2,
                          "marginal_sum_us_per_step": mtotal / 2}))
        print(f"{'marginal':>10} {'device':>10} {'count':>6}  kernel")
        for n, c, t in rows:
            print(f"{mt.get(n, 0.0) / 2:8.1f}us {t / 2:8.1f}us {c // 2:6d}x  {n}")
    llm.backend._graphs.clear()
    if comm:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["forward", "prefill", "engine"])
    ap.add_argument("--rows", type=int, default=8)
    ap.add_argument("--chunk", type=int, default=4096)
    ap.add_argument("--context", type=int, default=4096)
    ap.add_argument("--k", type=int, default=7)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--top", type=int, default=40)
    a = ap.parse_args()
    {"forward": cmd_forward, "prefill": cmd_prefill, "engine": cmd_engine}[a.mode](a)


if __name__ == "__main__":
    main()
