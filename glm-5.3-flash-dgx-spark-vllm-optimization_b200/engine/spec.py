"""Speculative-decoding control: adaptive K and the acceptance rules.

Adaptive K (the reference's launcher patch: EMA of acceptance over the set {4, 5, 7}, margin 1.0, alpha 0.25;
code/kit/launcher/start.sh:268, :581-587): after each verify step the EMA of accepted drafts is updated and the next
K is the smallest K of the set with K >= EMA + margin (the largest K when none qualifies).

Acceptance:
  greedy   accepted = length of the prefix of drafts equal to the target's argmax at each row (exact greedy
           decoding: the emitted sequence equals target-only greedy decoding)
  forced   all K drafts are accepted (benchmark mode: fixed tokens per step)
  sampled  rejection sampling with independent residual noise, standard or block verification (CUDA kernel
           csrc/sample.cu)
"""

from __future__ import annotations

from dataclasses import dataclass, field


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
