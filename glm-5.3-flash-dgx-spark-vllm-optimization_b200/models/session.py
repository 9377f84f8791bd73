"""A sequence driven directly on a ``Runtime`` (one request, contiguous cache slots): chunked prefill, verify
windows with commit, and greedy decode.  The engine (engine/) does the same for many requests with paged slots;
this class is the minimal driver used by tests, ``smoke()`` and the benchmark."""

from __future__ import annotations

import torch

from .runtime import Runtime


class Sequence:
    def __init__(self, rt: Runtime, index: int = 0):
        self.rt = rt
        self.index = index
        rc = rt.rc
        per_seq_blocks = rc.kv_slots // rc.block_size // rc.max_seqs
        if per_seq_blocks < 1:
            raise ValueError("kv_slots too small for max_seqs sequences")
        first = index * per_seq_blocks
        self.block_table = list(range(first, first + min(per_seq_blocks, rc.max_blocks)))
        self.capacity = len(self.block_table) * rc.block_size
        self.pos = 0
        self.cur = 0                   # which of the two KDA state buffers is committed

    def _slot(self, p: int) -> int:
        bs = self.rt.rc.block_size
        return self.block_table[p // bs] * bs + p % bs

    def _seq_desc(self, nrows: int):
        s_in = 2 * self.index + self.cur
        return (0, nrows, s_in, 2 * self.index + (1 - self.cur), self.index)

    def reset(self):
        self.pos = 0
        self.cur = 0
        i = self.index
        for S in getattr(self.rt, "S_pool", []):
            S[2 * i:2 * i + 2].zero_()
        for cp in getattr(self.rt, "conv_pool", []):
            cp[i].zero_()

    def stage(self, tokens, logit_rows):
        n = len(tokens)
        if self.pos + n > self.capacity:
            raise ValueError("sequence exceeds its cache capacity")
        pos = list(range(self.pos, self.pos + n))
        self.rt.stage(list(tokens), pos, [self._slot(p) for p in pos], [0] * n, [self._seq_desc(n)],
                      [self.block_table], logit_rows)

    @torch.no_grad()
    def prefill(self, tokens, chunk: int | None = None) -> torch.Tensor:
        """Run the prompt in chunks; returns the logits of the last prompt token [1, V_local]."""
        chunk = chunk or self.rt.rc.max_rows
        out = None
        for i in range(0, len(tokens), chunk):
            part = tokens[i:i + chunk]
            self.stage(part, [len(part) - 1])
            out = self.rt.forward(keep_window=False)
            self.cur = 1 - self.cur
            self.pos += len(part)
        return out

    @torch.no_grad()
    def verify(self, tokens) -> torch.Tensor:
        """A window of rows at the next positions (not committed): logits of every row."""
        n = len(tokens)
        self.stage(tokens, list(range(n)))
        self._window = n
        return self.rt.forward(keep_window=True)

    def commit(self, keep: int):
        n = self._window
        if not 1 <= keep <= n:
            raise ValueError("keep must be in 1..window")
        d = self._seq_desc(keep)
        self.rt.commit([d], replay=keep < n)
        self.cur = 1 - self.cur
        self.pos += keep

    @torch.no_grad()
    def decode_greedy(self, first_logits: torch.Tensor, n: int) -> list[int]:
        toks = []
        logits = first_logits
        for _ in range(n):
            t = int(torch.argmax(logits[-1]))
            toks.append(t)
            logits = self.verify([t])
            self.commit(1)
        return toks
