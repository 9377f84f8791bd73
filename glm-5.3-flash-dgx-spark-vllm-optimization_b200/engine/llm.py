"""The serving engine: continuous batching with chunked prefill, paged caches with prefix reuse, and speculative
decoding with a block drafter and adaptive K.

Per ``step()``:
  1. admit waiting requests (a request slot + pages; prefix-cache reuse where a KDA state checkpoint exists)
  2. prefill: the next chunk of each prefilling request (chunk ends aligned to the checkpoint interval, so the KDA
     state can be saved at page-aligned prefixes), several requests in one forward up to ``prefill_chunk`` rows;
     the request whose prompt completes samples its first token
  3. decode: every running request contributes a window [last token, K drafts]; one forward verifies all windows;
     greedy / forced / sampled acceptance; commit keeps the accepted rows (KDA replay when a window is cut); the
     drafter proposes the next K tokens; adaptive K updates per request
Reference behaviour: vLLM's V1 engine as configured by the reference (code/kit/launcher/start.sh:2666-2741), chunked
prefill aligned to KDA blocks (code/kit/launcher/overlay/patch_mamba_align_chunking.py), DFlash2 speculative decoding
with adaptive K (README.md:40, REPRODUCE.md:333).
"""

from __future__ import annotations

import hashlib
import itertools
import time
from array import array
from dataclasses import dataclass, field
from enum import Enum

import torch

from .kv_manager import KVManager, OutOfPages, SeqCache, StateSlots
from .spec import AdaptiveK, greedy_accept, rejection_sample_host


MAX_LOGPROBS = 20      # most alternatives per token a request may ask for (the OpenAI API's top_logprobs limit)


@dataclass
class SamplingParams:
    max_tokens: int = 64
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    seed: int | None = None
    stop_token_ids: tuple[int, ...] = ()
    ignore_eos: bool = False
    logprobs: int | None = None            # per emitted token: its log-probability and the top-n alternatives
                                           # (raw model distribution, before temperature and filters)


@dataclass
class EngineConfig:
    max_seqs: int = 4
    page_size: int = 64
    num_pages: int = 256
    max_model_len: int = 8192
    prefill_chunk: int = 8192
    speculative: bool = True
    k_set: tuple[int, ...] = (4, 5, 7)
    k_fixed: int | None = None
    ema_alpha: float = 0.25
    k_margin: float = 1.0
    force_accept: bool = False             # benchmark mode: every draft accepted
    block_verify: bool = False             # sampled requests: block verification instead of standard
    checkpoints: int = 0                   # KDA state checkpoint slots (prefix cache for hybrid state)
    checkpoint_pages: int = 8              # checkpoint interval in pages
    prefill_first: bool = True             # a step with waiting prefill runs it before decode
    mixed_prefill_chunk: int = 0           # > 0: prefill tokens per step while requests are decoding (bounds the
                                           # decode stall a newcomer causes; 0 = the whole prefill_chunk budget)
    cuda_graphs: bool = True
    vtrim_tau: float = 0.0                 # > 0: verify only the drafts before the first one whose drafter
                                           # confidence (max softmax probability) is below tau


class State(Enum):
    WAITING = 0
    PREFILL = 1
    RUNNING = 2
    FINISHED = 3


@dataclass
class Request:
    rid: str
    prompt: list[int]
    params: SamplingParams
    arrival: float = field(default_factory=time.time)
    state: State = State.WAITING
    output: list[int] = field(default_factory=list)
    cache: SeqCache = field(default_factory=SeqCache)
    slot: int = -1
    cur: int = 0
    pos: int = 0                            # tokens committed to the caches
    drafts: list[int] = field(default_factory=list)
    draft_probs: torch.Tensor | None = None   # sampled requests: q_i of each draft row [k, V]
    hidden: torch.Tensor | None = None
    adaptive: AdaptiveK | None = None
    first_token_time: float | None = None
    finish_reason: str | None = None
    cached_tokens: int = 0
    accepted: list = field(default_factory=list)
    logprobs: list = field(default_factory=list)    # per output token: (logprob, {token: logprob} top-n)
    _new_lp: list | None = None

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.output

    def token_view(self, extra: list[int] = ()) -> "TokenView":
        """prompt + output + extra without building the list (long contexts: the engine hashes only new pages)."""
        return TokenView((self.prompt, self.output, list(extra)))


class TokenView:
    """Read-only concatenation of token lists, sliced on demand.  The prefix cache hashes only the pages completed
    by a step, so a decode step at a 512k context copies a few pages instead of the whole prompt."""

    def __init__(self, parts):
        self.parts = parts

    def __len__(self) -> int:
        return sum(len(p) for p in self.parts)

    def __getitem__(self, sl: slice) -> list[int]:
        start, stop, step = sl.indices(len(self))
        assert step == 1, "contiguous slices only"
        out, base = [], 0
        for p in self.parts:
            n = len(p)
            lo, hi = max(start - base, 0), min(stop - base, n)
            if lo < hi:
                out.extend(p[lo:hi])
            base += n
            if base >= stop:
                break
        return out


@dataclass
class RequestOutput:
    rid: str
    new_tokens: list[int]
    finished: bool
    finish_reason: str | None
    output: list[int]
    new_logprobs: list | None = None      # aligned with new_tokens when the request asked for logprobs


class LLMEngine:
    def __init__(self, backend, cfg: EngineConfig, eos: tuple[int, ...] = ()):
        self.b = backend
        self.cfg = cfg
        self.eos = set(eos)
        self.kv = KVManager(cfg.num_pages, cfg.page_size, (cfg.max_model_len + cfg.page_size - 1) // cfg.page_size)
        self.slots = StateSlots(cfg.max_seqs, cfg.checkpoints)
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        self.done: dict[str, Request] = {}
        self._ids = itertools.count()
        self.metrics = {"prompt_tokens": 0, "generation_tokens": 0, "steps": 0, "spec_drafts": 0,
                        "spec_accepted": 0, "prefix_cached_tokens": 0, "requests_finished": 0, "vtrim_cut": 0,
                        "spec_windows": 0, "spec_accepted_per_pos": [0] * 16}
        # verify-trim records (drafted K, verified after the trim), most recent last
        import collections
        self.vtrim_records = collections.deque(maxlen=4096)

    # ------------------------------------------------------------------------------------------------ requests
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, rid: str | None = None) -> str:
        params = params or SamplingParams()
        if len(prompt) == 0:
            raise ValueError("empty prompt")
        if len(prompt) + params.max_tokens > self.cfg.max_model_len:
            raise ValueError(f"prompt + max_tokens exceeds max_model_len {self.cfg.max_model_len}")
        self.check_params(params)
        rid = rid or f"req-{next(self._ids)}"
        r = Request(rid, list(prompt), params)
        r.adaptive = AdaptiveK(self.cfg.k_set, self.cfg.ema_alpha, self.cfg.k_margin, fixed=self.cfg.k_fixed)
        self.waiting.append(r)
        self.metrics["prompt_tokens"] += len(prompt)
        return rid

    def check_params(self, params: SamplingParams) -> None:
        """Reject sampling fields that a step could not serve, before the request is queued: a bad value raised
        later inside ``step()`` (``topk`` over more alternatives than the vocabulary, say) would fail every request
        in flight, not just this one."""
        vocab = getattr(self.b, "vocab", None)
        if params.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if params.logprobs is not None:
            cap = MAX_LOGPROBS if vocab is None else min(MAX_LOGPROBS, vocab)
            if not 0 <= params.logprobs <= cap:
                raise ValueError(f"logprobs must be in [0, {cap}]")
        if params.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0.0 < params.top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if params.top_k < 0:
            raise ValueError("top_k must be >= 0")
        if vocab is not None and any(not 0 <= t < vocab for t in params.stop_token_ids):
            raise ValueError("stop_token_ids must be token ids of the vocabulary")

    def abort(self, rid: str) -> None:
        for q in (self.waiting, self.running):
            for r in q:
                if r.rid == rid:
                    r.finish_reason = "abort"
                    self._finish(r)
                    return

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ------------------------------------------------------------------------------------------------ admission
    def _admit(self) -> None:
        while self.waiting and self.slots.free:
            r = self.waiting[0]
            pids, hashes = self.kv.match_prefix(r.prompt[:-1])     # always recompute at least the last token
            start = 0
            ck = None
            if pids and self.cfg.checkpoints:
                # the longest cached prefix that also has a KDA state checkpoint
                for n in range(len(hashes), 0, -1):
                    ck = self.slots.find(hashes[n - 1])
                    if ck is not None and ck.tokens == n * self.cfg.page_size:
                        pids, hashes = pids[:n], hashes[:n]
                        start = n * self.cfg.page_size
                        break
                    ck = None
            if not self.kv.can_grow(SeqCache(pages=list(pids if start else [])), len(r.prompt) + 8):
                break
            self.waiting.pop(0)
            r.slot = self.slots.alloc()
            r.cur = 0
            self.b.reset_state(r.slot)
            if start:
                self.kv.adopt_prefix(r.cache, pids, hashes)
                self.b.load_state(ck.slot, r.slot, r.cur)
                r.pos = start
                r.cached_tokens = start
                self.metrics["prefix_cached_tokens"] += start
            r.state = State.PREFILL
            self.running.append(r)

    # ------------------------------------------------------------------------------------------------ step
    def step(self) -> list[RequestOutput]:
        self.metrics["steps"] += 1
        self._admit()
        outs: list[RequestOutput] = []
        prefill = [r for r in self.running if r.state == State.PREFILL]
        decode = [r for r in self.running if r.state == State.RUNNING]
        if prefill and (self.cfg.prefill_first or not decode):
            budget = self.cfg.prefill_chunk
            if decode and self.cfg.mixed_prefill_chunk > 0:
                budget = min(budget, self.cfg.mixed_prefill_chunk)
            outs += self._prefill_step(prefill, budget)
        decode = [r for r in self.running if r.state == State.RUNNING]
        if decode:
            outs += self._decode_step(decode)
        return outs

    def _rows(self, r: Request, tokens: list[int], pos0: int):
        from .backend import SeqRows
        n = len(tokens)
        self.kv.grow(r.cache, pos0 + n)
        positions = list(range(pos0, pos0 + n))
        return SeqRows(tokens, positions, [self.kv.slot(r.cache, p) for p in positions], array("i", r.cache.pages),
                       r.slot, r.cur)

    def _prefill_step(self, reqs: list[Request], budget: int | None = None) -> list[RequestOutput]:
        budget = self.cfg.prefill_chunk if budget is None else budget
        batch, ends = [], []
        interval = self.cfg.checkpoint_pages * self.cfg.page_size if self.cfg.checkpoints else 0
        for r in reqs:
            if budget <= 0:
                break
            remaining = len(r.prompt) - r.pos
            n = min(remaining, budget)
            if interval:
                # end the chunk on a checkpoint boundary when one lies inside it
                nxt = (r.pos // interval + 1) * interval
                if r.pos + n > nxt and nxt < len(r.prompt):
                    n = nxt - r.pos
            try:
                rows = self._rows(r, r.prompt[r.pos:r.pos + n], r.pos)
            except OutOfPages:
                break
            batch.append((r, rows))
            budget -= n
        if not batch:
            return []
        logit_rows, row = [], 0
        finishing = []
        for r, rows in batch:
            row += len(rows.tokens)
            if r.pos + len(rows.tokens) == len(r.prompt):
                logit_rows.append(row - 1)
                finishing.append((r, row - 1))
        logits = self.b.prefill([rows for _, rows in batch], logit_rows)
        outs = []
        for r, rows in batch:
            r.pos += len(rows.tokens)
            r.cur = 1 - r.cur
            self.kv.commit_tokens(r.cache, r.token_view(), r.pos)
            self._checkpoint(r)
        if finishing:
            toks = self._sample_rows(logits, [r for r, _ in finishing])
            want = [i for i, (r, _) in enumerate(finishing) if r.params.logprobs is not None]
            if want:
                lps = self._logprobs(logits[want], [toks[i] for i in want], [finishing[i][0] for i in want])
                for i, lp in zip(want, lps):
                    finishing[i][0]._new_lp = [lp]
            to_draft = []
            for i, (r, row_idx) in enumerate(finishing):
                r.state = State.RUNNING
                r.first_token_time = time.time()
                r.hidden = self.b.hidden(row_idx).clone()
                outs.append(self._emit(r, [toks[i]]))
                if r.state == State.RUNNING and self.cfg.speculative and self.b.drafter is not None:
                    to_draft.append(r)
            self._draft_many(to_draft)
        return outs

    def _sample_rows(self, logits: torch.Tensor, reqs: list[Request]) -> list[int]:
        """One token per row: greedy rows by argmax, sampled rows with temperature / top-k / top-p."""
        greedy = self.b.argmax(logits)
        out = []
        full = None
        for i, r in enumerate(reqs):
            p = r.params
            if p.temperature <= 0:
                out.append(greedy[i])
                continue
            if full is None:
                full = self.b.full_logits(logits).float()
            out.append(sample_token(full[i], p, seed_key(r, len(r.output))))
        return out

    def _draft_many(self, reqs: list[Request]) -> None:
        """Drafts of several requests: those with the same draft length share one drafter pass (one graph per
        (k, batch) in the backend) instead of one pass per request."""
        if len(reqs) <= 1 or not hasattr(self.b, "draft_batch"):
            for r in reqs:
                self._draft(r)
            return
        groups: dict[int, list[Request]] = {}
        for r in reqs:
            groups.setdefault(r.adaptive.current(), []).append(r)
        for k, rs in groups.items():
            if len(rs) == 1:
                self._draft(rs[0])
                continue
            drafts, lg = self.b.draft_batch([r.output[-1] for r in rs], [r.hidden for r in rs], k)
            for b, r in enumerate(rs):
                self._draft(r, (drafts[b], lg[b * k:(b + 1) * k]))

    def _draft(self, r: Request, drafted=None) -> None:
        k = r.adaptive.current()
        drafts, lg = drafted if drafted is not None else self.b.draft(r.output[-1], r.hidden, k)
        n = k
        if self.cfg.vtrim_tau > 0 and not self.cfg.force_accept:
            # verify trimming (the reference's n* rule, code/fork/glm53_spec_vtrim.py:11-23): rows past the first
            # low-confidence draft are unlikely to be accepted, so they are not verified
            conf = self.b.draft_confidence(lg[:k])
            n = next((i for i, c in enumerate(conf) if c < self.cfg.vtrim_tau), k)
            self.metrics["vtrim_cut"] += k - n
            self.vtrim_records.append((k, n))
        r.drafts = drafts[:n]
        r.draft_probs = None
        p = r.params
        if p.temperature > 0 and n and not self.cfg.force_accept:
            # probabilistic drafts: row i is drawn from q_i, the drafter's distribution after the request's
            # temperature / top-k / top-p, and q_i is what the verifier divides by (rows of the block drafter do not
            # depend on one another's tokens, so each q_i is a valid proposal on its own)
            q = torch.softmax(apply_filters(self.b.full_logits(lg[:n]).float() / p.temperature, p), -1)
            g = torch.Generator(device=q.device)
            g.manual_seed(lane_key(seed_key(r, len(r.output)), 1))        # a lane apart from the target's keys
            r.drafts = torch.multinomial(q, 1, generator=g).view(-1).tolist()
            r.draft_probs = q

    def _decode_step(self, reqs: list[Request]) -> list[RequestOutput]:
        spec = self.cfg.speculative and self.b.drafter is not None
        batch = []
        for r in list(reqs):
            window = [r.output[-1]] + (r.drafts if spec else [])
            try:
                batch.append((r, self._rows(r, window, r.pos)))
            except OutOfPages:
                r.finish_reason = "length"
                self._finish(r)
        if not batch:
            return []
        logits = self.b.verify([rows for _, rows in batch])
        greedy = self.b.argmax(logits)
        outs, keeps, row = [], [], 0
        for r, rows in batch:
            n_rows = len(rows.tokens)
            tgt = greedy[row:row + n_rows]
            drafts = rows.tokens[1:]
            if self.cfg.force_accept:
                n_acc = len(drafts)
                new = drafts + [tgt[-1]]
            elif r.params.temperature <= 0:
                n_acc = greedy_accept(drafts, tgt)
                new = drafts[:n_acc] + [tgt[n_acc]]
            else:
                n_acc, new = self._sampled_accept(r, logits[row:row + n_rows], drafts)
            keeps.append(n_acc + 1)
            r._new = new
            if r.params.logprobs is not None:
                r._new_lp = self._logprobs(logits[row:row + len(new)], new, [r] * len(new))
            r._last_row = row + n_acc
            row += n_rows
            if drafts:
                self.metrics["spec_drafts"] += len(drafts)
                self.metrics["spec_accepted"] += n_acc
                self.metrics["spec_windows"] += 1
                per_pos = self.metrics["spec_accepted_per_pos"]
                for i in range(min(n_acc, len(per_pos))):
                    per_pos[i] += 1
                r.accepted.append(n_acc)
                r.adaptive.update(n_acc)
        # a state checkpoint interval boundary strictly inside a sequence's kept rows splits its commit there, so
        # the recurrent state at the boundary can be saved for later prefix hits (multi-turn follow-ups)
        interval = self.cfg.checkpoint_pages * self.cfg.page_size if self.cfg.checkpoints else 0
        first, rest = list(keeps), []
        if interval:
            for i, ((r, _), keep) in enumerate(zip(batch, keeps)):
                bnd = (r.pos // interval + 1) * interval
                if bnd < r.pos + keep:
                    first[i] = bnd - r.pos
                    rest.append((i, first[i], keep - first[i]))
        self.b.commit(first)
        for (r, rows), keep, k1 in zip(batch, keeps, first):
            r.pos += k1
            r.cur = 1 - r.cur
            # the accepted drafts are not in r.output yet: hash the committed positions' own tokens
            self.kv.commit_tokens(r.cache, r.token_view(r._new[:keep - 1]), r.pos)
            self._checkpoint(r)
        if rest:
            self.b.commit_rest(rest)
            for i, _, n in rest:
                r = batch[i][0]
                r.pos += n
                r.cur = 1 - r.cur
                self.kv.commit_tokens(r.cache, r.token_view(r._new[:keeps[i] - 1]), r.pos)
                self._checkpoint(r)
        to_draft = []
        for (r, rows), keep in zip(batch, keeps):
            r.hidden = self.b.hidden(r._last_row).clone()
            outs.append(self._emit(r, r._new))
            if r.state == State.RUNNING and spec:
                to_draft.append(r)
        self._draft_many(to_draft)
        return outs

    def _checkpoint(self, r: Request) -> None:
        """Save the request's committed recurrent state when its committed length sits on a checkpoint boundary
        (a page-aligned prefix whose pages are in the prefix cache)."""
        interval = self.cfg.checkpoint_pages * self.cfg.page_size if self.cfg.checkpoints else 0
        if not interval or r.pos % interval or len(r.cache.hashes) < r.pos // self.cfg.page_size:
            return
        ck = self.slots.checkpoint_slot(r.cache.hashes[r.pos // self.cfg.page_size - 1], r.pos)
        if ck is not None:
            self.b.save_state(r.slot, r.cur, ck.slot)

    def _logprobs(self, logits: torch.Tensor, tokens: list[int], reqs: list[Request]) -> list:
        """(log-probability of each row's token, its top-n alternatives) from the rows' full logits."""
        lp = torch.log_softmax(self.b.full_logits(logits).float(), -1)
        n = max((r.params.logprobs or 0) for r in reqs)
        chosen = lp.gather(1, torch.tensor(tokens, device=lp.device).view(-1, 1)).view(-1).tolist()
        top = torch.topk(lp, n, -1) if n > 0 else None
        tv = top.values.tolist() if top is not None else None
        ti = top.indices.tolist() if top is not None else None
        out = []
        for i, r in enumerate(reqs):
            k = r.params.logprobs or 0
            out.append((chosen[i], {ti[i][j]: tv[i][j] for j in range(k)} if k else {}))
        return out

    def _sampled_accept(self, r: Request, logits: torch.Tensor, drafts: list[int]):
        """Rejection sampling of one request's window (CUDA kernel; standard or block verification)."""
        from ..ops import kernels as K
        p = r.params
        full = self.b.full_logits(logits).float()
        tp = torch.softmax(apply_filters(full / p.temperature, p), -1)
        k = len(drafts)
        if k == 0:
            return 0, [sample_token(full[0], p, seed_key(r, len(r.output)))]
        dp = r.draft_probs[:k]
        dev = tp.device
        if not tp.is_cuda:
            # host tensors (the CPU test backend): the same standard rule in PyTorch
            if self.cfg.block_verify:
                raise NotImplementedError("block verification runs in the CUDA kernel only")
            g = torch.Generator()
            g.manual_seed(lane_key(seed_key(r, len(r.output)), 2))
            return rejection_sample_host(tp, dp, drafts, g)
        acc = torch.zeros(1, dtype=torch.int32, device=dev)
        nxt = torch.zeros(1, k + 1, dtype=torch.int32, device=dev)
        K.C().rejection_sample(tp.view(1, k + 1, -1).contiguous(), dp.view(1, k, -1).contiguous(),
                               torch.tensor([drafts], dtype=torch.int32, device=dev),
                               int(p.seed if p.seed is not None else rid_key(r.rid)) & ((1 << 62) - 1),
                               torch.tensor([r.pos], dtype=torch.int64, device=dev), self.cfg.block_verify, acc, nxt,
                               None)
        n = int(acc.item())
        row = nxt[0].tolist()
        return n, row[:n + 1]

    # ------------------------------------------------------------------------------------------------ outputs
    def _emit(self, r: Request, new: list[int]) -> RequestOutput:
        emitted = []
        lp, r._new_lp = r._new_lp, None
        new_lp = [] if lp is not None else None
        for i, t in enumerate(new):
            emitted.append(t)
            r.output.append(t)
            if lp is not None:
                r.logprobs.append(lp[i])
                new_lp.append(lp[i])
            self.metrics["generation_tokens"] += 1
            if (t in self.eos and not r.params.ignore_eos) or t in r.params.stop_token_ids:
                r.finish_reason = "stop"
                break
            if len(r.output) >= r.params.max_tokens:
                r.finish_reason = "length"
                break
        if r.finish_reason is not None:
            self._finish(r)
        return RequestOutput(r.rid, emitted, r.state == State.FINISHED, r.finish_reason, list(r.output), new_lp)

    def _finish(self, r: Request) -> None:
        if r in self.running:
            self.running.remove(r)
        if r in self.waiting:
            self.waiting.remove(r)
        if r.slot >= 0:
            self.slots.release(r.slot)
            r.slot = -1
        self.kv.free(r.cache)
        r.state = State.FINISHED
        self.done[r.rid] = r
        self.metrics["requests_finished"] += 1

    # ------------------------------------------------------------------------------------------------ offline
    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None,
                 on_step=None) -> list[list[int]]:
        if not isinstance(params, list):
            params = [params or SamplingParams()] * len(prompts)
        rids = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        while any(rid not in self.done for rid in rids):
            outs = self.step()
            if on_step:
                on_step(outs)
        return [self.done[rid].output for rid in rids]


def rid_key(rid: str) -> int:
    """A key of a request id that is the same in every process (Python's str hash is salted per process, and the
    tensor-parallel ranks must draw the same samples for an unseeded request)."""
    return int.from_bytes(hashlib.blake2b(rid.encode(), digest_size=8).digest(), "little")


def seed_key(r: Request, index: int) -> int:
    base = r.params.seed if r.params.seed is not None else (rid_key(r.rid) & 0xFFFFFFFF)
    return (base * 1000003 + index) & ((1 << 63) - 1)


def lane_key(key: int, lane: int) -> int:
    """The seed of one independent use (lane) of a sampling key: the SplitMix64 finaliser (Steele, Lea, Flood 2014)
    of key + lane x the 64-bit golden-ratio increment. Every output bit depends on every input bit, so lanes differ in
    the low 32 bits too (the CPU generator keeps only those of a seed)."""
    m = (1 << 64) - 1
    z = (key + lane * 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return (z ^ (z >> 31)) & ((1 << 63) - 1)


def apply_filters(logits: torch.Tensor, p: SamplingParams) -> torch.Tensor:
    x = logits
    if p.top_k and p.top_k > 0:
        kth = torch.topk(x, min(p.top_k, x.shape[-1]), dim=-1).values[..., -1:]
        x = torch.where(x < kth, torch.full_like(x, float("-inf")), x)
    if p.top_p < 1.0:
        srt, idx = torch.sort(x, dim=-1, descending=True)
        cum = torch.softmax(srt, -1).cumsum(-1)
        drop = cum - torch.softmax(srt, -1) > p.top_p
        srt = torch.where(drop, torch.full_like(srt, float("-inf")), srt)
        x = torch.full_like(x, float("-inf")).scatter(-1, idx, srt)
    return x


def sample_token(logits: torch.Tensor, p: SamplingParams, key: int) -> int:
    x = apply_filters(logits / max(p.temperature, 1e-6), p)
    g = torch.Generator(device=x.device)
    g.manual_seed(key)
    probs = torch.softmax(x, -1)
    return int(torch.multinomial(probs, 1, generator=g).item())
