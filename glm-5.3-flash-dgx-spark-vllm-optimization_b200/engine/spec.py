"""Speculative-decoding control: adaptive K and the acceptance rules.

Adaptive K (the reference's launcher patch: EMA of acceptance over the set {4, 5, 7}, margin 1.0, alpha 0.25;
code/kit/launcher/start.sh:268, :581-587): after each verify step the EMA of accepted drafts is updated and the next
K is the smallest K of the set with K >= EMA + margin (the largest K when none qualifies).

Acceptance:
  greedy   accepted = length of the prefix of drafts equal to the target's argmax at each row (exact greedy
           decoding: the emitted sequence equals target-only greedy decoding)
  forced   all K drafts are accepted (benchmark mode: fixed tokens per step)
  sampled  rejection sampling with independent residual noise, standard or block verification (CUDA kernel
           csrc/sample.cu). Draft i is drawn from the drafter's own filtered distribution q_i (probabilistic draft
           sampling, as the reference's DFlash2 config runs it: code/kit/launcher/start.sh:2697-2706), and q_i is the
           distribution the verifier divides by; a greedy draft verified against q_i would bias the output.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class AdaptiveK:
    ks: tuple[int, ...] = (4, 5, 7)
    alpha: float = 0.25
    margin: float = 1.0
    ema: float | None = None
    fixed: int | None = None
    history: list = field(default_factory=list)

    def current(self) -> int:
        if self.fixed is not None:
            return self.fixed
        if self.ema is None:
            return max(self.ks)
        for k in sorted(self.ks):
            if k >= self.ema + self.margin:
                return k
        return max(self.ks)

    def update(self, accepted: int) -> int:
        self.ema = accepted if self.ema is None else self.alpha * accepted + (1 - self.alpha) * self.ema
        self.history.append(accepted)
        return self.current()


def greedy_accept(drafts: list[int], target: list[int]) -> int:
    """Number of leading drafts equal to the target's greedy tokens (target has len(drafts) + 1 entries)."""
    n = 0
    while n < len(drafts) and drafts[n] == target[n]:
        n += 1
    return n


def rejection_sample_host(tp: torch.Tensor, dp: torch.Tensor, drafts: list[int],
                          gen: torch.Generator) -> tuple[int, list[int]]:
    """Standard speculative sampling (Leviathan et al. 2023, Chen et al. 2023) on host tensors, the rule the CUDA
    kernel applies per row: draft x_i ~ q_i is accepted with probability min(1, p_i(x_i) / q_i(x_i)); the first
    rejection emits a token from the residual max(0, p_i - q_i) (renormalised) and ends the window; when every draft
    is accepted the bonus token comes from p_k. tp [k+1, V] and dp [k, V] are probabilities. Returns (accepted,
    emitted tokens)."""
    for i, x in enumerate(drafts):
        u = float(torch.rand((), generator=gen, dtype=torch.float64))
        if u * float(dp[i, x]) < float(tp[i, x]):
            continue
        resid = (tp[i].double() - dp[i].double()).clamp_min(0)
        s = float(resid.sum())
        nxt = int(torch.multinomial(resid / s if s > 0 else tp[i].double(), 1, generator=gen))
        return i, list(drafts[:i]) + [nxt]
    k = len(drafts)
    return k, list(drafts) + [int(torch.multinomial(tp[k].double(), 1, generator=gen))]
