"""Teacher-forced KL / NLL harness (the role of the reference's klh, code/operator/klh/klh.py:1-45): two logit providers
read the same token sequences; per position the KL divergence KL(P_a || P_b) of their next-token distributions and
each provider's negative log-likelihood of the actual next token are collected, with block-bootstrap confidence
intervals (blocks of consecutive positions, so correlated neighbours do not shrink the interval) and an A/A noise
floor (provider a against itself on a second pass: nonzero only if the provider is not deterministic).

Providers:
  reference   the fp32 CPU oracle (models/reference.py), one token at a time
  runtime     the GPU runtime: the sequence prefilled in windows of `logit_rows` rows with every row's logits
              (the same kernels as decode windows)

  python -m glm53.utils.klh --model tiny --a runtime --b reference --seqs 2 --len 96
"""

from __future__ import annotations

import argparse
import json

import torch


def kl_rows(la: torch.Tensor, lb: torch.Tensor) -> torch.Tensor:
    """KL(softmax(la) || softmax(lb)) per row (fp64)."""
    pa = torch.log_softmax(la.double(), -1)
    pb = torch.log_softmax(lb.double(), -1)
    return (pa.exp() * (pa - pb)).sum(-1)


def nll_rows(l: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return -torch.log_softmax(l.double(), -1).gather(-1, target[:, None]).squeeze(-1)


def block_bootstrap(x: torch.Tensor, block: int = 16, reps: int = 400, seed: int = 0) -> tuple[float, float]:
    """95 % interval of the mean of x by resampling blocks of `block` consecutive values."""
    n = x.numel()
    if n == 0:
        return (float("nan"), float("nan"))
    nb = max(1, n // block)
    blocks = [x[i * block:(i + 1) * block] for i in range(nb)]
    g = torch.Generator().manual_seed(seed)
    means = []
    for _ in range(reps):
        idx = torch.randint(0, nb, (nb,), generator=g)
        means.append(torch.cat([blocks[i] for i in idx.tolist()]).mean().item())
    means.sort()
    return means[int(0.025 * reps)], means[int(0.975 * reps) - 1]


def reference_provider(weights_cpu):
    from ..models.reference import ReferenceModel
    m = ReferenceModel(weights_cpu)

    def run(tokens: list[int]) -> torch.Tensor:
        m.reset()
        return torch.stack([m.step(t).float().flatten() for t in tokens])
    return run


def runtime_provider(weights_gpu, window: int = 16, max_len: int = 4096):
    """Logits of every position, the sequence run through the GPU runtime in windows of `window` rows: up to 16
    rows take the decode kernels (GEMV, per-row attention), from 64 rows on the prefill kernels (tcgen05 GEMM,
    chunked KDA)."""
    from ..models.runtime import Runtime, RuntimeConfig
    from ..models.session import Sequence
    blocks = (max_len + 63) // 64
    rc = RuntimeConfig(max_rows=window, max_seqs=1, kv_slots=64 * blocks, block_size=64, max_blocks=blocks,
                       logit_rows=window)
    rt = Runtime(weights_gpu, rc)

    def run(tokens: list[int]) -> torch.Tensor:
        seq = Sequence(rt)
        seq.reset()
        out = []
        for i in range(0, len(tokens), window):
            part = tokens[i:i + window]
            seq.stage(part, list(range(len(part))))
            out.append(rt.forward(keep_window=False).float().cpu())
            seq.cur = 1 - seq.cur
            seq.pos += len(part)
        return torch.cat(out)
    return run


def compare(run_a, run_b, seqs: list[list[int]], block: int = 16) -> dict:
    kls, nll_a, nll_b, aa, agree = [], [], [], [], []
    for toks in seqs:
        la, lb = run_a(toks).cpu(), run_b(toks).cpu()
        la2 = run_a(toks).cpu()
        tgt = torch.tensor(toks[1:])
        kls.append(kl_rows(la[:-1], lb[:-1]))
        aa.append(kl_rows(la[:-1], la2[:-1]))
        nll_a.append(nll_rows(la[:-1], tgt))
        nll_b.append(nll_rows(lb[:-1], tgt))
        agree.append((la[:-1].argmax(-1) == lb[:-1].argmax(-1)).double())
    kl, a_a = torch.cat(kls), torch.cat(aa)
    na, nb = torch.cat(nll_a), torch.cat(nll_b)
    return {"positions": kl.numel(), "kl_mean": kl.mean().item(), "kl_ci95": block_bootstrap(kl, block),
            "kl_max": kl.max().item(), "aa_kl_mean": a_a.mean().item(), "nll_a": na.mean().item(),
            "nll_b": nb.mean().item(), "dnll_ci95": block_bootstrap(na - nb, block),
            "top1_agree": torch.cat(agree).mean().item()}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--a", default="runtime", choices=["runtime", "reference"])
    ap.add_argument("--b", default="reference", choices=["runtime", "reference"])
    ap.add_argument("--seqs", type=int, default=2)
    ap.add_argument("--len", type=int, default=96)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    from ..config import config_by_name
    from ..models import weights as W
    cfg = config_by_name(args.model)
    w_cpu = W.prepare(W.RandomSource(cfg, seed=0, device="cpu"), cfg, device=torch.device("cpu"))
    providers = {}
    if "reference" in (args.a, args.b):
        providers["reference"] = reference_provider(w_cpu)
    if "runtime" in (args.a, args.b):
        providers["runtime"] = runtime_provider(W.to_device(w_cpu, torch.device("cuda", 0)))
    g = torch.Generator().manual_seed(args.seed)
    seqs = [torch.randint(16, cfg.vocab, (args.len,), generator=g).tolist() for _ in range(args.seqs)]
    res = compare(providers[args.a], providers[args.b], seqs)
    res.update({"a": args.a, "b": args.b, "model": args.model})
    print(json.dumps(res))


if __name__ == "__main__":
    main()
