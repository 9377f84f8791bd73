"""Greedy sampling over a vocabulary-parallel lm_head: per-rank argmax kernel, then (tensor parallel) an
all-gather of the per-rank (value, id) pairs and the global maximum (ties -> lower id)."""

from __future__ import annotations

import torch

from . import kernels as K


class GreedySampler:
    def __init__(self, rows: int, world: int, vocab_offset: int, comm=None, device="cuda"):
        self.world, self.offset, self.comm = world, vocab_offset, comm
        self.val = torch.zeros(rows, dtype=torch.float32, device=device)
        self.idx = torch.zeros(rows, dtype=torch.int32, device=device)
        if world > 1:
            self.gval = torch.zeros(world * rows, dtype=torch.float32, device=device)
            self.gidx = torch.zeros(world * rows, dtype=torch.int32, device=device)
        self.out = torch.zeros(rows, dtype=torch.int32, device=device)

    def __call__(self, logits: torch.Tensor) -> torch.Tensor:
        R = logits.shape[0]
        K.C().argmax_rows(logits, self.offset, self.val[:R], self.idx[:R])
        if self.world == 1:
            return self.idx[:R]
        self.comm.all_gather(self.gval[:self.world * R], self.val[:R])
        self.comm.all_gather(self.gidx[:self.world * R], self.idx[:R])
        v = self.gval[:self.world * R].view(self.world, R)
        i = self.gidx[:self.world * R].view(self.world, R)
        best = v.max(0).values
        cand = torch.where(v == best, i, torch.full_like(i, 2 ** 31 - 1))
        torch.amin(cand, 0, out=self.out[:R])
        return self.out[:R]
