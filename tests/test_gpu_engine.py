"""The engine on the GPU with the tiny proxy: greedy speculative decoding emits exactly the tokens of greedy
decoding without speculation (per-row kernels are independent of window composition), concurrent requests, and a
prefix-cache hit (KDA checkpoint + shared pages) reproduces the cold-start output of the same chunking.  (Runs with
different prefill chunk boundaries are not compared token for token: chunk size selects between the chunked and the
recurrent KDA kernels and between the prefill and decode MoE kernels, whose fp32 summation orders differ.)"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _llm(**kw):
    from glm53.api.offline import LLM, LLMOptions
    opts = dict(model="tiny", max_seqs=4, max_model_len=1024, prefill_chunk=128, page_size=64, checkpoints=4)
    opts.update(kw)
    return LLM(LLMOptions(**opts))


def _prompts(n, length, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(16, 4096, (length + 7 * i,), generator=g).tolist() for i in range(n)]


def test_spec_greedy_equals_plain_greedy():
    from glm53.engine.llm import SamplingParams
    prompts = _prompts(3, 150)
    sp = SamplingParams(max_tokens=40, ignore_eos=True)
    plain = _llm(speculative=False).engine.generate(prompts, sp)
    spec_llm = _llm(speculative=True)
    spec = spec_llm.engine.generate(prompts, sp)
    assert spec == plain
    m = spec_llm.engine.metrics
    assert m["spec_drafts"] > 0


def test_forced_acceptance_and_text_api():
    from glm53.engine.llm import SamplingParams
    llm = _llm(speculative=True, k_fixed=7, force_accept=True)
    out = llm.generate(["hello B200"], SamplingParams(max_tokens=33, ignore_eos=True))
    assert len(out[0]["token_ids"]) == 33
    assert isinstance(out[0]["text"], str)


def test_prefix_cache_hit_reproduces_output():
    from glm53.engine.llm import SamplingParams
    base = _prompts(1, 300, seed=3)[0]
    # the engine saves KDA checkpoints every 8 pages (512 tokens) by default -> use a 64-token interval here
    llm2 = _llm(speculative=False, checkpoints=4)
    llm2.engine.cfg.checkpoint_pages = 1
    a2 = llm2.engine.generate([base], SamplingParams(max_tokens=16, ignore_eos=True))[0]
    b = llm2.engine.generate([base], SamplingParams(max_tokens=16, ignore_eos=True))[0]
    assert llm2.engine.metrics["prefix_cached_tokens"] >= 256
    assert a2 == b


def test_decode_checkpoints_split_commits_stay_exact():
    """With a state checkpoint every page, decode windows that straddle a page boundary commit in two parts (the
    KDA recurrence replayed up to the boundary, the state saved, then the rest of the kept rows); greedy speculative
    decoding must still emit exactly the tokens of plain greedy decoding, and a follow-up request that repeats the
    prompt and answer resumes from a checkpoint inside the answer."""
    from glm53.engine.llm import SamplingParams
    prompt = _prompts(1, 100, seed=7)[0]
    sp = SamplingParams(max_tokens=90, ignore_eos=True)
    # the same checkpoint interval in both runs: prefill chunks end at checkpoint boundaries (64 + 36 rows here), and
    # a different chunking would select different kernels (the 64-row chunk takes the decode-path MoE kernels)
    plain_llm = _llm(speculative=False, checkpoints=8)
    plain_llm.engine.cfg.checkpoint_pages = 1
    plain = plain_llm.engine.generate([prompt], sp)[0]
    llm = _llm(speculative=True, checkpoints=8)
    llm.engine.cfg.checkpoint_pages = 1
    spec = llm.engine.generate([prompt], sp)[0]
    assert spec == plain
    follow = prompt + spec + [11, 12, 13]
    before = llm.engine.metrics["prefix_cached_tokens"]
    llm.engine.generate([follow], SamplingParams(max_tokens=4, ignore_eos=True))
    assert llm.engine.metrics["prefix_cached_tokens"] - before > len(prompt)


def test_kv_budget_in_bytes_sizes_the_page_pool():
    """kv_cache_bytes sets the page pool from the configuration's bytes per token, which equals what the runtime
    allocates per token slot."""
    from glm53.utils.longctx import kv_bytes_per_token
    budget = 4 << 20
    llm = _llm(kv_cache_bytes=budget)
    bpt = llm.cfg.kv_bytes_per_token()
    assert abs(kv_bytes_per_token(llm.backend.rt) - bpt) <= 1
    assert llm.engine.cfg.num_pages == int(budget // (bpt * 64))


def test_batched_drafter_equals_single_drafts():
    """Several requests drafted in one pass (rows of request b at [b k, (b+1) k), attention and dynamic convolutions
    inside each block) give each request's logits bit for bit as its own single-request pass."""
    from glm53.config import tiny_config
    from glm53.models import weights as W
    from glm53.models.drafter import BlockDrafter
    cfg = tiny_config()
    w = W.prepare(W.RandomSource(cfg, seed=0, device="cuda"), cfg, device="cuda")
    d = BlockDrafter(cfg, w, device="cuda", max_batch=4)
    g = torch.Generator(device="cuda").manual_seed(3)
    hid = [(torch.randn(cfg.hidden, device="cuda", generator=g)).to(torch.bfloat16) for _ in range(3)]
    last = [17, 401, 3999]
    for k in (4, 7):
        d.stage_batch(last, hid, k)
        batched = d.run_batch(3, k).clone()
        for b in range(3):
            d.stage(last[b], hid[b])
            single = d.run(k).clone()
            assert torch.equal(batched[b * k:(b + 1) * k], single), (k, b)
