"""A deterministic stand-in for the GPU backend (CPU only): next token = f(last three tokens of the sequence); the
drafter proposes f except at every third draft position (so acceptance varies).  It keeps per-slot token histories
with the same commit / checkpoint contract as the real backend, so the engine's scheduling, paging, prefix reuse and
speculative verification can be tested without a GPU."""

from __future__ import annotations

import torch

V = 512


def next_tok(hist):
    a = hist[-1] if len(hist) > 0 else 0
    b = hist[-2] if len(hist) > 1 else 0
    c = hist[-3] if len(hist) > 2 else 0
    return (a * 31 + b * 17 + c * 7 + 11) % (V - 16) + 16


def onehot(t):
    x = torch.full((V,), -5.0)
    x[t] = 5.0
    return x


class FakeBackend:
    def __init__(self, max_seqs=8, checkpoints=4, drafter_error_every=3):
        self.hist = {s: [] for s in range(max_seqs)}       # committed tokens per state slot
        self.ck = {}
        self.drafter = self
        self.err = drafter_error_every
        self.calls = {"prefill": 0, "verify": 0, "commit": 0, "commit_rest": 0, "draft": 0, "save": 0, "load": 0}
        self._pending = []
        self._hidden = []

    # prefill: rows are committed immediately
    def prefill(self, seqs, logit_rows):
        self.calls["prefill"] += 1
        out, self._hidden = [], []
        for s in seqs:
            h = self.hist[s.state_slot]
            assert s.positions[0] == len(h), (s.positions[0], len(h))
            for t in s.tokens:
                h.append(t)
                out.append(onehot(next_tok(h)))
                self._hidden.append(torch.tensor(list(h[-3:]) + [0] * (3 - len(h[-3:])), dtype=torch.float32))
        return torch.stack([out[i] for i in logit_rows]) if logit_rows else None

    def verify(self, seqs):
        self.calls["verify"] += 1
        out, self._hidden, self._pending = [], [], []
        for s in seqs:
            h = list(self.hist[s.state_slot])
            assert s.positions[0] == len(h)
            for t in s.tokens:
                h.append(t)
                out.append(onehot(next_tok(h)))
                self._hidden.append(torch.tensor(h[-3:], dtype=torch.float32))
            self._pending.append((s.state_slot, s.tokens))
        return torch.stack(out)

    def commit(self, keeps):
        self.calls["commit"] += 1
        for (slot, toks), k in zip(self._pending, keeps):
            self.hist[slot] += toks[:k]

    def commit_rest(self, parts):
        self.calls["commit_rest"] += 1
        for i, off, n in parts:
            slot, toks = self._pending[i]
            assert len(self.hist[slot]) >= off
            self.hist[slot] += toks[off:off + n]

    def hidden(self, row):
        return self._hidden[row]

    def argmax(self, logits):
        return torch.argmax(logits, -1).tolist()

    def full_logits(self, logits):
        return logits

    def draft(self, last_token, hidden, k):
        self.calls["draft"] += 1
        h = [int(x) for x in hidden.tolist()][:-1] + [last_token]
        # hidden holds the last three committed tokens ending at the row that produced last_token
        h = [int(x) for x in hidden.tolist()] + [last_token]
        drafts = []
        for i in range(k):
            t = next_tok(h)
            if self.err and (i + 1) % self.err == 0:
                t = (t + 1) % V
            drafts.append(t)
            h.append(t)
        return drafts, torch.stack([onehot(t) for t in drafts])

    def draft_confidence(self, logits):
        """softmax max-probability of the one-hot-like rows, lowered for rows the drafter got wrong"""
        p = torch.softmax(logits.float(), -1).max(-1).values
        return [float(x) * (0.1 if self.err and (i + 1) % self.err == 0 else 1.0) for i, x in enumerate(p)]

    def save_state(self, slot, cur, ck):
        self.calls["save"] += 1
        self.ck[ck] = list(self.hist[slot])

    def load_state(self, ck, slot, cur):
        self.calls["load"] += 1
        self.hist[slot] = list(self.ck[ck])

    def reset_state(self, slot):
        self.hist[slot] = []


def reference_greedy(prompt, n):
    h = list(prompt)
    out = []
    for _ in range(n):
        t = next_tok(h)
        out.append(t)
        h.append(t)
    return out
