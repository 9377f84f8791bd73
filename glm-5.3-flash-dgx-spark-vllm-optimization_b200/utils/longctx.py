"""Long-context serving measurements (MAX_MODEL_LEN up to 1M tokens): KV token capacity of a paged pool of a given
size, and decode ms/step against the context length, through the public engine API.

For every context length a request with uniform random token ids is prefilled through the engine (chunked, the
same path as any prompt), then `--steps` speculative decode steps (K drafts, acceptance forced) are timed with CUDA
events, max over ranks.  With `--concurrency C`, C such requests decode together (one verify window of C x (K+1)
rows per step).  The KV bytes per token are read from the runtime's own cache allocation (fp8 latent + scale + rope
key per MLA layer and the pooled fp8 index keys + scales; raw index keys are kept only in a per-sequence tail ring,
not per token), so the capacity figure is what this engine stores, per GPU (the latent and index caches are
replicated over tensor-parallel ranks).

    python -m glm53.utils.longctx --contexts 4096 32768 131072 --steps 8
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m glm53.utils.longctx --contexts 131072 524288

Reference counterparts: the operator's long-context probe (code/operator/longctx_probe.py) and the 1M-token
MAX_MODEL_LEN deployment (REPRODUCE.md:307).
"""

from __future__ import annotations

import argparse
import json
import sys
import time

import torch


def kv_bytes_per_token(rt) -> int:
    """Device bytes of the per-token caches of one runtime (all MLA/DSA layers), per token slot."""
    slots = rt.kv[0].shape[0] if getattr(rt, "kv", None) else 0
    if not slots:
        return 0
    total = 0
    for name in ("kv", "kv_scale", "kpe", "pool", "pool_scale"):
        for t in getattr(rt, name, []):
            total += t.numel() * t.element_size()
    return total // slots


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--contexts", type=int, nargs="+", default=[4096, 32768, 131072])
    ap.add_argument("--concurrency", type=int, nargs="+", default=[1])
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--k", type=int, default=7)
    ap.add_argument("--kv-gib", type=float, default=15.0, help="pool size for the capacity figure")
    ap.add_argument("--prefill-chunk", type=int, default=8192)
    ap.add_argument("--model", default="full")
    args = ap.parse_args(argv)

    from ..api.offline import LLM, LLMOptions
    from ..engine.llm import SamplingParams, State
    from ..parallel import dist as D

    rank, local, world = D.init()
    comm = D.NcclComm() if world > 1 else None
    K = args.k
    rows = K + 1
    results = []
    for conc in args.concurrency:
        for ctx in args.contexts:
            # requests that finish their prefill first decode (K + 1 tokens per engine step) while the others are
            # still prefilling: budget those steps too, or the early ones reach max_tokens before the timed steps
            prefill_steps = -(-conc * ctx // args.prefill_chunk) + conc
            max_len = ctx + rows * (args.steps + args.warmup + 8 + prefill_steps) + 64
            llm = LLM(LLMOptions(model=args.model, max_seqs=conc, max_model_len=max_len,
                                 prefill_chunk=args.prefill_chunk, speculative=True, k_fixed=K, force_accept=True,
                                 checkpoints=0, cuda_graphs=True), comm=comm, rank=rank, world=world)
            eng, cfg = llm.engine, llm.cfg
            gen = torch.Generator().manual_seed(ctx + conc)
            stream = torch.cuda.current_stream()

            def sync():
                if comm:
                    comm.barrier()
                torch.cuda.synchronize()

            sync()
            t0 = time.perf_counter()
            rids = [eng.add_request(torch.randint(0, cfg.vocab, (ctx,), generator=gen).tolist(),
                                    SamplingParams(max_tokens=max_len - ctx - 8, ignore_eos=True))
                    for _ in range(conc)]
            nsteps = 0
            stalled = False
            while not (len(eng.running) == conc and all(r.state == State.RUNNING for r in eng.running)):
                if not eng.running and not eng.waiting:
                    # every request ended before decoding (the KV pool or a request limit cut it short): nothing
                    # left to time; every rank sees the same engine state, so all leave together
                    stalled = True
                    break
                eng.step()
                nsteps += 1
                if rank == 0 and nsteps % 16 == 0:
                    print(f"# prefill: {nsteps} steps, {time.perf_counter() - t0:.1f} s, running "
                          f"{len(eng.running)}, waiting {len(eng.waiting)}", file=sys.stderr, flush=True)
            sync()
            prefill_s = time.perf_counter() - t0
            if stalled:
                if rank == 0:
                    print(json.dumps({"context": ctx, "concurrency": conc, "tp": world,
                                      "error": "requests finished during prefill (KV pool or request limits)",
                                      "requests_finished": eng.metrics["requests_finished"]}), flush=True)
                llm.backend._graphs.clear()
                del llm, eng
                torch.cuda.empty_cache()
                continue
            for _ in range(args.warmup):
                eng.step()
            sync()
            n0 = sum(len(r.output) for r in eng.running)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.steps):
                eng.step()
            e1.record(stream)
            sync()
            ms = e0.elapsed_time(e1)
            ms = comm.max_scalar(ms) if comm else ms
            emitted = sum(len(r.output) for r in eng.running) - n0
            rt = llm.backend.rt
            bpt = kv_bytes_per_token(rt)
            res = {"context": ctx, "concurrency": conc, "tp": world, "ms_per_step": ms / args.steps,
                   "tok_s": emitted / (ms / 1e3), "tokens_per_step": emitted / args.steps,
                   "prefill_s_wall": prefill_s, "prefill_tok_s_wall": conc * ctx / prefill_s,
                   "kv_bytes_per_token": bpt,
                   "kv_capacity_tokens": int(args.kv_gib * 2 ** 30 // bpt) if bpt else None,
                   "kv_pool_gib_assumed": args.kv_gib}
            results.append(res)
            if rank == 0:
                print(json.dumps(res), flush=True)
            llm.backend._graphs.clear()
            del llm, eng, rt
            torch.cuda.empty_cache()
    if comm:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return results


if __name__ == "__main__":
    main()
