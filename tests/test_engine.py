"""Engine logic on CPU with a deterministic fake backend: exact greedy speculative decoding, forced acceptance,
adaptive K, chunked prefill, paging and prefix reuse with KDA checkpoints, concurrency, limits."""

import pytest
import torch

from glm53.engine.kv_manager import KVManager, OutOfPages, PageAllocator, SeqCache, page_hash
from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams
from glm53.engine.spec import AdaptiveK, greedy_accept
from tests.fake_backend import FakeBackend, reference_greedy


def _engine(**kw):
    cfg = EngineConfig(**{"max_seqs": 4, "page_size": 16, "num_pages": 128, "max_model_len": 1024,
                          "prefill_chunk": 48, "cuda_graphs": False, **kw})
    return LLMEngine(FakeBackend(max_seqs=cfg.max_seqs, checkpoints=cfg.checkpoints), cfg)


@pytest.mark.parametrize("spec", [False, True])
def test_greedy_output_equals_target_greedy(spec):
    e = _engine(speculative=spec)
    prompt = list(range(20, 120))
    out = e.generate([prompt], SamplingParams(max_tokens=40))[0]
    assert out == reference_greedy(prompt, 40)
    if spec:
        m = e.metrics
        assert 0 < m["spec_accepted"] < m["spec_drafts"]     # the drafter is wrong every third position


def test_forced_acceptance_emits_k_plus_one():
    e = _engine(force_accept=True, k_fixed=7)
    e.add_request(list(range(20, 60)), SamplingParams(max_tokens=64))
    e.step()                                                # prefill + first token (+ first decode window)
    n0 = len(e.running[0].output) if e.running else 64
    e.step()
    n1 = len(e.running[0].output) if e.running else 64
    assert n1 - n0 == 8


def test_adaptive_k():
    ak = AdaptiveK((4, 5, 7), alpha=0.25, margin=1.0)
    assert ak.current() == 7
    for _ in range(20):
        ak.update(1)
    assert ak.current() == 4
    for _ in range(40):
        ak.update(7)
    assert ak.current() == 7
    assert greedy_accept([1, 2, 3], [1, 2, 9, 4]) == 2


def test_concurrent_requests_and_chunked_prefill():
    e = _engine(max_seqs=3, prefill_chunk=32)
    prompts = [list(range(30 + i, 130 + 3 * i)) for i in range(5)]
    outs = e.generate(prompts, [SamplingParams(max_tokens=10 + 5 * i) for i in range(5)])
    for p, o, i in zip(prompts, outs, range(5)):
        assert o == reference_greedy(p, 10 + 5 * i)
    assert e.metrics["requests_finished"] == 5
    assert not e.running and not e.waiting
    assert e.kv.alloc.num_free == 128                      # every page back (free or evictable)


def test_prefix_reuse_with_state_checkpoint():
    e = _engine(checkpoints=4, checkpoint_pages=2, page_size=16)
    shared = list(range(40, 40 + 96))                       # 3 checkpoint intervals of 32 tokens
    a = e.generate([shared + [7, 8, 9]], SamplingParams(max_tokens=8))[0]
    b_prompt = shared + [5, 6]
    b = e.generate([b_prompt], SamplingParams(max_tokens=8))[0]
    assert b == reference_greedy(b_prompt, 8)
    assert e.metrics["prefix_cached_tokens"] == 96
    assert e.b.calls["load"] == 1
    assert a == reference_greedy(shared + [7, 8, 9], 8)


def test_stop_tokens_and_max_len():
    e = _engine()
    prompt = list(range(20, 50))
    ref = reference_greedy(prompt, 30)
    out = e.generate([prompt], SamplingParams(max_tokens=30, stop_token_ids=(ref[5],)))[0]
    assert out == ref[:6]
    with pytest.raises(ValueError):
        e.add_request(list(range(1000)), SamplingParams(max_tokens=100))


def test_page_allocator_prefix_cache_and_eviction():
    pa = PageAllocator(4, 8)
    p0, p1 = pa.alloc(), pa.alloc()
    h0 = page_hash(None, list(range(8)))
    pa.register(p0, h0)
    pa.release(p0)
    pa.release(p1)
    assert pa.num_free == 4
    assert pa.lookup(h0) == p0
    got = [pa.alloc() for _ in range(4)]                   # the cached page is evicted last
    assert p0 in got and pa.stats["evictions"] == 1
    with pytest.raises(OutOfPages):
        pa.alloc()


def test_kv_manager_slots():
    kv = KVManager(16, 8, 4)
    sc = SeqCache()
    kv.grow(sc, 20)
    assert len(sc.pages) == 3
    assert kv.slot(sc, 9) == sc.pages[1] * 8 + 1
    with pytest.raises(OutOfPages):
        kv.grow(sc, 40)
    kv.free(sc)
    assert kv.alloc.num_free == 16


def test_step_tracer_records(tmp_path):
    """Per-step trace records (host phases, collectives) from the tracer on the fake backend."""
    import json
    from glm53.utils.trace import StepTracer, rank_skew
    from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams

    class Comm:
        def all_reduce(self, t):
            return t
    eng = LLMEngine(FakeBackend(), EngineConfig(max_seqs=2, page_size=16, num_pages=64, max_model_len=512,
                                                prefill_chunk=32, cuda_graphs=False))
    comm = Comm()
    tr = StepTracer(str(tmp_path / "trace"), 0).attach(eng, comm)
    eng.add_request(list(range(20, 60)), SamplingParams(max_tokens=5))
    while eng.has_work():
        eng.step()
        comm.all_reduce(torch.zeros(4))
    tr.close()
    recs = [json.loads(l) for l in open(tr.path)]
    assert len(recs) >= 2 and all(r["rank"] == 0 for r in recs)
    assert any("backend.prefill" in r["phases_ms"] for r in recs)
    assert rank_skew([tr.path])[0]["start_skew_ms"] == 0.0


def test_profiler_signal_and_memory_report(tmp_path):
    import os
    import signal
    from glm53.utils.runtime_helpers import install_profiler_signal, memory_report
    eng = LLMEngine(FakeBackend(), EngineConfig(max_seqs=2, page_size=16, num_pages=64, max_model_len=512,
                                                prefill_chunk=32, cuda_graphs=False))
    ctl = install_profiler_signal(eng, steps=2, out_dir=str(tmp_path))
    os.kill(os.getpid(), signal.SIGUSR2)
    eng.add_request(list(range(20, 40)), SamplingParams(max_tokens=6))
    while eng.has_work():
        eng.step()
    assert os.path.exists(ctl.last_path)
    assert isinstance(memory_report(), dict)


def test_vtrim_cuts_verify_rows_keeps_output():
    """Verify trimming: drafts after the first low-confidence one are not verified; greedy output unchanged."""
    prompt = list(range(30, 70))
    outs = {}
    for tau in (0.0, 0.5):
        eng = LLMEngine(FakeBackend(), EngineConfig(max_seqs=2, page_size=16, num_pages=64, max_model_len=512,
                                                    prefill_chunk=32, cuda_graphs=False, k_fixed=7, vtrim_tau=tau))
        outs[tau] = eng.generate([prompt], SamplingParams(max_tokens=30))[0]
        if tau > 0:
            assert eng.metrics["vtrim_cut"] > 0 and len(eng.vtrim_records) > 0
    assert outs[0.0] == outs[0.5] == reference_greedy(prompt, 30)


@pytest.mark.parametrize("force", [False, True])
def test_decoded_pages_are_hashed_from_their_tokens(force):
    """Pages filled during speculative decoding enter the prefix cache under the hash of the tokens they hold (the
    accepted drafts are committed before they are emitted): the whole committed sequence matches afterwards."""
    e = _engine(speculative=True, force_accept=force, k_fixed=7 if force else None)
    prompt = list(range(30, 70))
    out = e.generate([prompt], SamplingParams(max_tokens=90, ignore_eos=True))[0]
    committed = prompt + out[:-1]                         # the last emitted token has no cache entry yet
    pids, _ = e.kv.match_prefix(committed)
    assert len(pids) == len(committed) // 16


@pytest.mark.parametrize("force", [False, True])
def test_decode_checkpoints_serve_follow_up_turns(force):
    """State checkpoints are also taken where decoding crosses a checkpoint boundary (the window's commit is split
    there), so a follow-up request that repeats prompt + answer resumes inside the answer and still produces the
    target's greedy continuation."""
    e = _engine(speculative=True, force_accept=force, k_fixed=7 if force else None, checkpoints=8,
                checkpoint_pages=1)
    prompt = list(range(30, 70))
    out = e.generate([prompt], SamplingParams(max_tokens=70, ignore_eos=True))[0]
    assert e.b.calls["commit_rest"] > 0 or force         # windows straddled boundaries
    follow = prompt + out + [5, 6, 7]
    before = e.metrics["prefix_cached_tokens"]
    out2 = e.generate([follow], SamplingParams(max_tokens=20, ignore_eos=True))[0]
    hit = e.metrics["prefix_cached_tokens"] - before
    assert hit >= (len(prompt) + len(out) - 1) // 16 * 16 - 16 and hit > len(prompt)
    if force:
        assert out2[:1] == reference_greedy(follow, 1)   # forced acceptance emits drafts: only the first is target's
    else:
        assert out2 == reference_greedy(follow, 20)


def test_mixed_prefill_chunk_caps_prefill_beside_decodes():
    """With mixed_prefill_chunk set, a newcomer's prompt is prefilled at most that many tokens per step while other
    requests decode (their per-step stall stays bounded), and the whole budget is used when nothing decodes; the
    outputs are unchanged."""
    e = _engine(speculative=False, mixed_prefill_chunk=16, prefill_chunk=64)
    a = e.add_request(list(range(20, 50)), SamplingParams(max_tokens=40))
    e.step()                                       # a: the whole 30-token prompt (nothing decodes yet), then a decode
    assert e.running[0].pos >= 30
    b = e.add_request(list(range(100, 200)), SamplingParams(max_tokens=8))
    positions = []
    for _ in range(3):
        e.step()
        rb = next(r for r in e.running if r.rid == b)
        positions.append(rb.pos)
    assert positions == [16, 32, 48]
    while e.has_work():
        e.step()
    assert e.done[a].output == reference_greedy(list(range(20, 50)), 40)
    assert e.done[b].output == reference_greedy(list(range(100, 200)), 8)


@pytest.mark.parametrize("spec", [False, True])
def test_logprobs_follow_each_emitted_token(spec):
    """logprobs=n: every emitted token carries its log-probability under the model's raw distribution and the top-n
    alternatives, with speculative windows (several tokens per step) and without."""
    import math
    from tests.fake_backend import next_tok, onehot
    eng = _engine(speculative=spec)
    prompt = list(range(20, 50))
    rid = eng.add_request(prompt, SamplingParams(max_tokens=17, logprobs=2, ignore_eos=True))
    while rid not in eng.done:
        eng.step()
    r = eng.done[rid]
    assert len(r.logprobs) == len(r.output) == 17
    hist = list(prompt)
    for t, (lp, top) in zip(r.output, r.logprobs):
        ref = torch.log_softmax(onehot(next_tok(hist)), -1)
        assert math.isclose(lp, ref[t].item(), abs_tol=1e-5)
        assert len(top) == 2 and max(top, key=top.get) == t == next_tok(hist)
        hist.append(t)
    rid = eng.add_request(prompt, SamplingParams(max_tokens=5))
    while rid not in eng.done:
        eng.step()
    assert eng.done[rid].logprobs == []


def test_token_view_slices_match_the_concatenated_list():
    """The prefix cache hashes pages from a lazy view of prompt + output + accepted drafts: every contiguous slice
    equals the same slice of the materialised list, and committing through the view publishes the same hashes."""
    import random
    from glm53.engine.llm import TokenView
    from glm53.engine.kv_manager import page_hash
    rng = random.Random(0)
    parts = ([rng.randrange(1000) for _ in range(130)], [rng.randrange(1000) for _ in range(7)], [1, 2, 3])
    full = parts[0] + parts[1] + parts[2]
    v = TokenView(parts)
    assert len(v) == len(full)
    for _ in range(200):
        a = rng.randrange(0, len(full) + 5)
        b = rng.randrange(a, len(full) + 10)
        assert v[a:b] == full[a:b]
    ps, h_list, h_view, prev_l, prev_v = 16, [], [], None, None
    for i in range(len(full) // ps):
        prev_l = page_hash(prev_l, full[i * ps:(i + 1) * ps])
        prev_v = page_hash(prev_v, v[i * ps:(i + 1) * ps])
        h_list.append(prev_l)
        h_view.append(prev_v)
    assert h_list == h_view
