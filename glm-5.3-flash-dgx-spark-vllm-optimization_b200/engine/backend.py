"""Model backend of the engine: the GPU runtime (target + block drafter + samplers) behind a small interface that
the scheduler drives.  One backend per rank; under tensor parallelism every rank runs the same engine decisions
and the backend's collectives keep the ranks in lock step."""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.drafter import BlockDrafter
from ..models.runtime import Graphed, Runtime, RuntimeConfig
from ..ops import kernels as K
from ..ops.sampling import GreedySampler


@dataclass
class SeqRows:
    """One sequence's rows in a forward."""
    tokens: list[int]
    positions: list[int]
    slots: list[int]
    block_table: list[int]
    state_slot: int
    cur: int                         # committed KDA buffer parity of this request


class GPUBackend:
    def __init__(self, weights, rc: RuntimeConfig, comm=None, drafter: bool = True, cuda_graphs: bool = True,
                 checkpoints: int = 0):
        self.w = weights
        self.cfg = weights.cfg
        self.rt = Runtime(weights, rc, comm=comm)
        self.comm = comm
        self.world = weights.world
        dev = weights.device
        self.sampler = GreedySampler(rc.logit_rows, self.world, weights.rank * weights.head.n, comm, dev)
        self.drafter = BlockDrafter(self.cfg, weights, device=dev, max_batch=rc.max_seqs) if drafter else None
        self.draft_sampler = GreedySampler(8 * rc.max_seqs, self.world, weights.rank * weights.head.n, comm, dev)
        self.cuda_graphs = cuda_graphs
        self._graphs: dict = {}
        self.vocab = self.cfg.vocab
        # KDA state checkpoints (prefix cache): copies of every KDA layer's state and conv window
        self.ck_S = [torch.zeros((checkpoints,) + S.shape[1:], dtype=S.dtype, device=dev) for S in
                     getattr(self.rt, "S_pool", [])] if checkpoints else []
        self.ck_conv = [torch.zeros((checkpoints,) + cp.shape[1:], dtype=cp.dtype, device=dev) for cp in
                        getattr(self.rt, "conv_pool", [])] if checkpoints else []
        if rc.max_rows >= K.GEMM_MIN_M:
            # widening scratch of the largest fp8 projection used at large M (allocated before any capture)
            big = max(lw.kda.in_proj.w.numel() if lw.kda is not None else lw.mla.o_proj.w.numel()
                      for lw in weights.layers)
            K.reserve_gemm_scratch(big, dev)

    # ---------------------------------------------------------------------------------------------------------
    def _stage(self, seqs: list[SeqRows], logit_rows: list[int]):
        ids, pos, slots, row_seq, descs, tables = [], [], [], [], [], []
        for b, s in enumerate(seqs):
            descs.append((len(ids), len(s.tokens), 2 * s.state_slot + s.cur, 2 * s.state_slot + 1 - s.cur,
                          s.state_slot))
            ids += s.tokens
            pos += s.positions
            slots += s.slots
            row_seq += [b] * len(s.tokens)
            tables.append(s.block_table)
        self.rt.stage(ids, pos, slots, row_seq, descs, tables, logit_rows)
        return descs

    @torch.no_grad()
    def prefill(self, seqs: list[SeqRows], logit_rows: list[int]):
        """A prefill chunk (every row kept). Returns logits of ``logit_rows`` [n, V_local]."""
        self._stage(seqs, logit_rows)
        return self.rt.forward(keep_window=False, logits=bool(logit_rows))

    @torch.no_grad()
    def verify(self, seqs: list[SeqRows]):
        """A decode / verify window (rows are kept by ``commit``). Returns logits of every row."""
        R = sum(len(s.tokens) for s in seqs)
        descs = self._stage(seqs, list(range(R)))
        self._last_descs = descs
        b = self.rt.batch
        key = (R, b.B, b.max_rows_per_seq)
        if not self.cuda_graphs:
            return self.rt.forward(R, keep_window=True)
        g = self._graphs.get(key)
        if g is None:
            g = Graphed(lambda: self.rt.forward(R, keep_window=True))
            self._graphs[key] = g
        return g()

    @torch.no_grad()
    def commit(self, keeps: list[int]):
        descs = [(d[0], k, d[2], d[3], d[4]) for d, k in zip(self._last_descs, keeps)]
        replay = any(k < d[1] for d, k in zip(self._last_descs, keeps))
        self.rt.commit(descs, replay=replay)

    @torch.no_grad()
    def commit_rest(self, parts: list[tuple[int, int, int]]):
        """After commit(): commit n further rows (from row `offset` of the window) of sequence i of the last window,
        for each (i, offset, n), continuing from the state the first commit left in the other buffer."""
        descs = []
        for i, off, n in parts:
            d = self._last_descs[i]
            descs.append((d[0] + off, n, d[3], d[2], d[4]))
        self.rt.commit(descs, replay=True)

    def hidden(self, row: int) -> torch.Tensor:
        return self.rt.hidden[row]

    @torch.no_grad()
    def argmax(self, logits: torch.Tensor) -> list[int]:
        out = self.sampler(logits).tolist()          # synchronises: kernel error words can be read now
        if self.rt.px is not None:
            self.rt.px.check()
        return out

    @torch.no_grad()
    def full_logits(self, logits: torch.Tensor) -> torch.Tensor:
        """Vocabulary-parallel logits gathered to [n, V] on every rank."""
        if self.world == 1:
            return logits
        n, vl = logits.shape
        out = torch.empty(self.world * n * vl, dtype=logits.dtype, device=logits.device)
        self.comm.all_gather(out, logits.contiguous().view(-1))
        return out.view(self.world, n, vl).permute(1, 0, 2).reshape(n, self.world * vl)

    @torch.no_grad()
    def draft(self, last_token: int, hidden: torch.Tensor, k: int):
        """K draft tokens (greedy) and their logits [k, V_local]."""
        self.drafter.stage(int(last_token), hidden)
        if not self.cuda_graphs:
            lg = self.drafter.run(k)
        else:
            # one CUDA graph per draft length: the drafter's dozen small launches replay without host overhead
            g = self._graphs.get(("draft", k))
            if g is None:
                g = Graphed(lambda: self.drafter.run(k))
                self._graphs[("draft", k)] = g
            lg = g()
        return self.draft_sampler(lg).tolist(), lg

    @torch.no_grad()
    def draft_batch(self, last_tokens: list[int], hiddens: list[torch.Tensor], k: int):
        """K draft tokens (greedy) of several requests in one drafter pass (one CUDA graph per (k, batch)): per
        request its drafts, and the logits [B k, V_local] (request b's rows at [b k, (b+1) k))."""
        B = len(last_tokens)
        self.drafter.stage_batch(last_tokens, hiddens, k)
        if not self.cuda_graphs:
            lg = self.drafter.run_batch(B, k)
        else:
            g = self._graphs.get(("draft", k, B))
            if g is None:
                g = Graphed(lambda: self.drafter.run_batch(B, k))
                self._graphs[("draft", k, B)] = g
            lg = g()
        toks = self.draft_sampler(lg).tolist()
        return [toks[b * k:(b + 1) * k] for b in range(B)], lg

    @torch.no_grad()
    def draft_confidence(self, logits: torch.Tensor) -> list[float]:
        """Max softmax probability of each draft row over the whole (vocabulary-parallel) logits: each rank's
        (max, sum exp(l - max)) pairs are gathered and combined, p_max = 1 / sum_j s_j exp(m_j - M)."""
        lg = logits.float()
        m = lg.max(-1).values
        st = (lg - m[:, None]).exp().sum(-1)
        if self.world > 1:
            both = torch.stack([m, st]).flatten()
            out = torch.empty(self.world * both.numel(), device=both.device)
            self.comm.all_gather(out, both)
            g = out.view(self.world, 2, -1)
            M = g[:, 0].max(0).values
            S = (g[:, 1] * (g[:, 0] - M).exp()).sum(0)
        else:
            S = st
        return (1.0 / S).tolist()

    # ---------------------------------------------------------------------------------------------------------
    def save_state(self, state_slot: int, cur: int, ck: int) -> None:
        for S, cS in zip(self.rt.S_pool, self.ck_S):
            cS[ck].copy_(S[2 * state_slot + cur])
        for cp, ccp in zip(self.rt.conv_pool, self.ck_conv):
            ccp[ck].copy_(cp[state_slot])

    def load_state(self, ck: int, state_slot: int, cur: int) -> None:
        for S, cS in zip(self.rt.S_pool, self.ck_S):
            S[2 * state_slot + cur].copy_(cS[ck])
        for cp, ccp in zip(self.rt.conv_pool, self.ck_conv):
            cp[state_slot].copy_(ccp[ck])

    def reset_state(self, state_slot: int) -> None:
        for S in self.rt.S_pool:
            S[2 * state_slot:2 * state_slot + 2].zero_()
        for cp in self.rt.conv_pool:
            cp[state_slot].zero_()
