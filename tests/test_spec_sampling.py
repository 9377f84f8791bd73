"""Sampled speculative decoding through the engine on CPU: with a soft target (a Markov chain over four tokens) and a
soft block drafter whose argmax often disagrees with the target, the tokens the engine emits follow the target's
distribution exactly (chi-square over the joint of three generated tokens), because each draft is drawn from the
drafter's own filtered distribution and verified against that distribution. The host rejection rule is also shown to
be biased when a greedy draft is verified against the drafter's softmax, the failure the probabilistic drafts avoid."""

import itertools

import pytest
import torch

from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams
from glm53.engine.spec import rejection_sample_host
from tests.fake_backend import V, FakeBackend

scipy_stats = pytest.importorskip("scipy.stats")

SUPPORT = [16, 17, 18, 19]
_g = torch.Generator().manual_seed(7)
TARGET = torch.randn(4, 4, generator=_g) * 1.2              # target logits over SUPPORT given the last token
DRAFT = torch.randn(4, 8, 4, generator=_g) * 1.2            # drafter logits given (last token, draft row)


def _row(logits4):
    x = torch.full((V,), -1e4)
    x[SUPPORT] = logits4
    return x


def target_probs(last):
    return torch.softmax(TARGET[SUPPORT.index(last)], -1)


class SoftBackend(FakeBackend):
    """Target: next token ~ softmax(TARGET[last]) over SUPPORT. Drafter: row i ~ softmax(DRAFT[last][i]), proposed
    greedily (its argmax), as the real drafter proposes; the engine resamples sampled requests' drafts."""

    def prefill(self, seqs, logit_rows):
        self.calls["prefill"] += 1
        out, self._hidden = [], []
        for s in seqs:
            h = self.hist[s.state_slot]
            for t in s.tokens:
                h.append(t)
                out.append(_row(TARGET[SUPPORT.index(t)]) if t in SUPPORT else _row(torch.zeros(4)))
                self._hidden.append(torch.zeros(3))
        return torch.stack([out[i] for i in logit_rows]) if logit_rows else None

    def verify(self, seqs):
        self.calls["verify"] += 1
        out, self._hidden, self._pending = [], [], []
        for s in seqs:
            for t in s.tokens:
                out.append(_row(TARGET[SUPPORT.index(t)]))
                self._hidden.append(torch.zeros(3))
            self._pending.append((s.state_slot, s.tokens))
        return torch.stack(out)

    def draft(self, last_token, hidden, k):
        self.calls["draft"] += 1
        lg = torch.stack([_row(DRAFT[SUPPORT.index(last_token), i]) for i in range(k)])
        return torch.argmax(lg, -1).tolist(), lg


def _expected_joint(first_last):
    p = {}
    for a, b, c in itertools.product(SUPPORT, repeat=3):
        p[(a, b, c)] = float(target_probs(first_last)[SUPPORT.index(a)] * target_probs(a)[SUPPORT.index(b)]
                             * target_probs(b)[SUPPORT.index(c)])
    return p


def _chi2_pvalue(counts, expected, n):
    keys = sorted(expected)
    obs = [counts.get(k, 0) for k in keys]
    tot = sum(expected.values())
    exp = [expected[k] / tot * n for k in keys]
    assert sum(obs) == n
    return float(scipy_stats.chisquare(obs, exp).pvalue)


def test_engine_sampled_speculative_decoding_is_lossless():
    n = 3000
    cfg = EngineConfig(max_seqs=64, page_size=16, num_pages=256, max_model_len=64, prefill_chunk=4096,
                       cuda_graphs=False, k_fixed=3)
    eng = LLMEngine(SoftBackend(max_seqs=64, checkpoints=0), cfg)
    prompt = [16, 17, 18]
    params = [SamplingParams(max_tokens=3, temperature=1.0, seed=10_000 + i, ignore_eos=True) for i in range(n)]
    outs = eng.generate([prompt] * n, params)
    counts = {}
    for o in outs:
        counts[tuple(o)] = counts.get(tuple(o), 0) + 1
    assert eng.metrics["spec_windows"] > 0 and 0 < eng.metrics["spec_accepted"] < eng.metrics["spec_drafts"]
    assert _chi2_pvalue(counts, _expected_joint(prompt[-1]), n) > 1e-4


def test_greedy_draft_against_drafter_softmax_is_biased():
    """The host rule with q = softmax(drafter) but the draft fixed at q's argmax: the first emitted token no longer
    follows p (the bias that drawing drafts from q removes); drawn from q it does."""
    p = torch.tensor([[0.5, 0.3, 0.2], [1 / 3, 1 / 3, 1 / 3]])
    q = torch.tensor([[0.2, 0.7, 0.1]])
    n = 20_000
    g = torch.Generator().manual_seed(1)
    greedy, drawn = [0, 0, 0], [0, 0, 0]
    for _ in range(n):
        _, toks = rejection_sample_host(p, q, [1], g)
        greedy[toks[0]] += 1
        x = int(torch.multinomial(q[0], 1, generator=g))
        _, toks = rejection_sample_host(p, q, [x], g)
        drawn[toks[0]] += 1
    exp = [float(v) * n for v in p[0]]
    assert scipy_stats.chisquare(drawn, exp).pvalue > 1e-4
    assert scipy_stats.chisquare(greedy, exp).pvalue < 1e-6


def test_seed_lanes_differ_in_the_bits_the_cpu_generator_keeps():
    """The CPU generator seeds from the low 32 bits only: the lanes of one key, and the keys of consecutive
    positions, must differ there (a flip of a high bit would give the draft and residual draws one stream)."""
    from glm53.engine.llm import lane_key, rid_key
    keys = [k * 1000003 + i for k in (0, 7, 10_000) for i in range(64)]
    low = {lane_key(k, lane) & 0xFFFFFFFF for k in keys for lane in (1, 2)}
    assert len(low) == 2 * len(keys)
    a = torch.Generator().manual_seed(lane_key(5, 1))
    b = torch.Generator().manual_seed(lane_key(5, 2))
    assert not torch.equal(torch.rand(8, generator=a), torch.rand(8, generator=b))
    assert rid_key("cmpl-1") == rid_key("cmpl-1") != rid_key("cmpl-2")
