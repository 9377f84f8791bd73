"""Quality probes of a serving configuration (the roles of the reference's operator probes: the short/long quality
probe code/kit/tools/quality_probe.py:1-9 and quality_long.py:1-5, the decode-vs-prefill consistency probe
code/kit/tools/kpool_decode_consistency.py:1-21 and the concurrency probe code/kit/tools/conc_quality_probe.py:1-30).
They run in-process on the engine and runtime of this package instead of through an HTTP server:

  run      fixed prompts: greedy completions through the engine (speculative decode on) and teacher-forced top-k
           log-probabilities of every prompt position through the prefill kernels; saved as JSON.  Run once per
           configuration (e.g. per arm of an environment A/B)
  compare  two saved runs: identical completions and the first divergent token; per-position KL over a partition
           of the vocabulary (one cell per token either run saved, one cell for the rest; each run's unsaved mass
           shared evenly over its unsaved tokens), mean / p95 / max, top-1 agreement
  dvp      decode vs prefill on the same sequences: every position's logits from decode windows (GEMV, per-row
           attention, recurrent KDA: the decode kernels) against prefill chunks (tcgen05 GEMM, chunked KDA, tensor-core
           attention); KL and top-1 per position bucket
  conc     concurrency: each prompt decoded alone, then all prompts decoded together in one engine; greedy token
           agreement and first divergence per stream (the engine's paged slots, per-request KDA state and indexer
           keys must not leak between requests), and speculative against plain greedy decoding

    python -m glm53.utils.quality_probe run --out a.json --model tiny
    python -m glm53.utils.quality_probe compare a.json b.json
    python -m glm53.utils.quality_probe dvp --model tiny --len 512
    python -m glm53.utils.quality_probe conc --model tiny --streams 4 --gen 64

The prompts are seeded random token ids (the weights are random-init unless a checkpoint directory is given, so text
carries no more meaning than ids); the same seed gives the same prompts in every run.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

BUCKETS = (0, 128, 512, 1024, 4096)


def topk_logprobs(logits: torch.Tensor, k: int) -> list[dict]:
    """Per row {token id: log-probability} of the k most likely tokens."""
    lp = torch.log_softmax(logits.double(), -1)
    v, i = lp.topk(k, -1)
    return [{int(a): float(b) for a, b in zip(ii.tolist(), vv.tolist())} for ii, vv in zip(i, v)]


def topk_kl(pa: dict, pb: dict, vocab: int) -> float:
    """KL(A || B) at one position, estimated from each run's saved top-k {token: log-probability} over a vocabulary
    of `vocab` tokens.

    The vocabulary is partitioned into one cell per token saved by either run, plus one cell for every other token.
    A run's probability of a cell:
    - a token it saved: the exponential of the saved log-probability;
    - any other token: an equal share of the mass it did not save, 1 - sum(exp(saved)), spread over its unsaved
      tokens (a token that only the other run kept thus gets this run's tail share);
    - the remaining cell: that share times the number of tokens in it.
    The statistic is the KL divergence of A's cell distribution from B's. It is non-negative. It is the exact KL
    when both runs saved the whole vocabulary, and it shrinks towards 0 as the runs agree on their top tokens."""
    union = sorted(set(pa) | set(pb))

    def cells(p: dict) -> torch.Tensor:
        lp = torch.tensor([p[t] for t in p], dtype=torch.float64)
        tail = max(0.0, 1.0 - float(lp.exp().sum()))
        share = tail / (vocab - len(p)) if vocab > len(p) else 0.0
        v = [math.exp(p[t]) if t in p else share for t in union]
        v.append(share * (vocab - len(union)))
        return torch.tensor(v, dtype=torch.float64)

    a, b = cells(pa), cells(pb)
    a, b = a / a.sum(), b / b.sum()                     # saved values may carry rounding: renormalise
    m = a > 0
    return float((a[m] * (a[m].log() - b[m].clamp_min(1e-300).log())).sum())


def top1(p: dict) -> int:
    """The most likely saved token (lowest id among ties)."""
    best = max(p.values())
    return min(t for t, v in p.items() if v == best)


def first_divergence(a: list[int], b: list[int]) -> int | None:
    for j, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return j
    return None if len(a) == len(b) else min(len(a), len(b))


def summarize(kls: list[float]) -> dict:
    if not kls:
        return {"n": 0}
    s = sorted(kls)
    return {"n": len(s), "kl_mean": sum(s) / len(s), "kl_p95": s[min(len(s) - 1, int(0.95 * len(s)))],
            "kl_max": s[-1]}


def compare_runs(A: dict, B: dict, start: int = 0) -> dict:
    """Statistics of two saved runs (same prompts)."""
    vocab = A.get("vocab") or B.get("vocab")
    if not vocab:
        raise ValueError("saved runs carry no vocabulary size (re-run `quality_probe run`)")
    same, divs = 0, []
    for ca, cb in zip(A["completions"], B["completions"]):
        d = first_divergence(ca, cb)
        same += d is None
        if d is not None:
            divs.append(d)
    kls, agree, n = [], 0, 0
    for ta, tb in zip(A["prompt_logprobs"], B["prompt_logprobs"]):
        for pa, pb in list(zip(ta, tb))[start:]:
            pa = {int(k): v for k, v in pa.items()}
            pb = {int(k): v for k, v in pb.items()}
            kls.append(topk_kl(pa, pb, vocab))
            agree += top1(pa) == top1(pb)
            n += 1
    out = {"decode_identical": same, "decode_streams": len(A["completions"]),
           "first_divergence": divs, "prefill": summarize(kls), "top1_agree": agree / n if n else None}
    return out


def prompts(vocab: int, n: int, length: int, seed: int) -> list[list[int]]:
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(16, vocab, (length,), generator=g).tolist() for _ in range(n)]


def _llm(model: str, max_seqs: int, max_len: int, speculative: bool = True, chunk: int = 512):
    from ..api.offline import LLM, LLMOptions
    return LLM(LLMOptions(model=model, max_seqs=max_seqs, max_model_len=max_len, prefill_chunk=chunk,
                          speculative=speculative, cuda_graphs=True))


def greedy(llm, ps: list[list[int]], gen: int) -> list[list[int]]:
    from ..engine.llm import SamplingParams
    return llm.engine.generate(ps, SamplingParams(max_tokens=gen, temperature=0.0, ignore_eos=True))


def cmd_run(args) -> dict:
    from ..utils.klh import runtime_provider
    llm = _llm(args.model, args.prompts, args.len + args.gen + 64)
    ps = prompts(llm.cfg.vocab, args.prompts, args.len, args.seed)
    comps = greedy(llm, ps, args.gen)
    w = llm.weights
    del llm
    torch.cuda.empty_cache()
    run = runtime_provider(w, window=args.chunk, max_len=args.len + 64)
    lps = [topk_logprobs(run(p)[:-1], args.topk) for p in ps]
    res = {"model": args.model, "seed": args.seed, "len": args.len, "gen": args.gen, "topk": args.topk,
           "vocab": int(w.cfg.vocab),
           "completions": comps, "prompt_logprobs": [[{str(k): v for k, v in d.items()} for d in t] for t in lps]}
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f)
    return {"saved": args.out, "prompts": len(ps), "positions": sum(len(t) for t in lps)}


def cmd_dvp(args) -> dict:
    from ..config import config_by_name
    from ..models import weights as W
    from ..utils.klh import kl_rows, runtime_provider
    cfg = config_by_name(args.model)
    dev = torch.device("cuda", torch.cuda.current_device())
    w = W.prepare(W.RandomSource(cfg, seed=0, device=dev), cfg, device=dev)
    dec = runtime_provider(w, window=args.window, max_len=args.len + 64)
    pre = runtime_provider(w, window=args.chunk, max_len=args.len + 64)
    per = {b: [] for b in BUCKETS}
    agree = []
    for p in prompts(cfg.vocab, args.prompts, args.len, args.seed):
        ld, lp = dec(p).cpu(), pre(p).cpu()
        kl = kl_rows(ld, lp)
        agree.append((ld.argmax(-1) == lp.argmax(-1)).double())
        for j, v in enumerate(kl.tolist()):
            b = max(x for x in BUCKETS if x <= j)
            per[b].append(v)
    return {"mode": "dvp", "model": args.model, "decode_window": args.window, "prefill_chunk": args.chunk,
            "buckets": {str(b): summarize(v) for b, v in per.items() if v},
            "top1_agree": torch.cat(agree).mean().item()}


def cmd_conc(args) -> dict:
    max_len = args.len + args.gen + 64
    llm = _llm(args.model, args.streams, max_len)
    ps = prompts(llm.cfg.vocab, args.streams, args.len, args.seed)
    solo = [greedy(llm, [p], args.gen)[0] for p in ps]
    conc = greedy(llm, ps, args.gen)
    del llm
    torch.cuda.empty_cache()
    plain_llm = _llm(args.model, 1, max_len, speculative=False)
    plain = [greedy(plain_llm, [p], args.gen)[0] for p in ps]
    d_conc = [first_divergence(a, b) for a, b in zip(solo, conc)]
    d_spec = [first_divergence(a, b) for a, b in zip(solo, plain)]
    tok = lambda xs, ys: sum(sum(x == y for x, y in zip(a, b)) for a, b in zip(xs, ys)) / sum(map(len, xs))
    return {"mode": "conc", "model": args.model, "streams": args.streams, "gen": args.gen,
            "conc_identical": sum(d is None for d in d_conc), "conc_first_divergence": d_conc,
            "conc_token_agree": tok(solo, conc),
            "spec_identical": sum(d is None for d in d_spec), "spec_first_divergence": d_spec,
            "spec_token_agree": tok(solo, plain)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    for name in ("run", "dvp", "conc"):
        s = sub.add_parser(name)
        s.add_argument("--model", default="tiny")
        s.add_argument("--seed", type=int, default=0)
        s.add_argument("--len", type=int, default=256)
        s.add_argument("--prompts", type=int, default=4)
        s.add_argument("--chunk", type=int, default=128)
        if name == "run":
            s.add_argument("--gen", type=int, default=64)
            s.add_argument("--topk", type=int, default=20)
            s.add_argument("--out", default="")
        if name == "dvp":
            s.add_argument("--window", type=int, default=8)
        if name == "conc":
            s.add_argument("--streams", type=int, default=4)
            s.add_argument("--gen", type=int, default=64)
    c = sub.add_parser("compare")
    c.add_argument("a")
    c.add_argument("b")
    c.add_argument("--start", type=int, default=0, help="first prompt position scored")
    args = ap.parse_args(argv)
    if args.cmd == "compare":
        with open(args.a) as fa, open(args.b) as fb:
            res = compare_runs(json.load(fa), json.load(fb), args.start)
    else:
        res = {"run": cmd_run, "dvp": cmd_dvp, "conc": cmd_conc}[args.cmd](args)
    print(json.dumps(res), flush=True)
    return res


if __name__ == "__main__":
    main()
