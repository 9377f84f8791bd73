"""Serving probes on CPU with the fake backend: the stall probe records the incumbent's steps around a newcomer's
prefill and a smaller mixed-prefill cap spreads that prefill over more steps; the prefix-cache probe serves the
follow-up turn's shared head from the cache and the perturbed cold prompt from nothing."""

from glm53.engine.llm import EngineConfig, LLMEngine
from glm53.utils import serve_probe as SP
from tests.fake_backend import FakeBackend


def _engine(**kw):
    cfg = EngineConfig(**{"max_seqs": 2, "page_size": 16, "num_pages": 256, "max_model_len": 1024,
                          "prefill_chunk": 256, "cuda_graphs": False, "k_fixed": 3, **kw})
    return LLMEngine(FakeBackend(max_seqs=2, checkpoints=cfg.checkpoints), cfg)


def test_stall_probe_counts_prefill_steps_per_cap():
    inc, new = list(range(20, 84)), [17 + (i * 7) % 400 for i in range(600)]
    res = {}
    for cap in (0, 64):
        res[cap] = SP.stall(_engine(mixed_prefill_chunk=cap), inc, new, gen=200, join_after=3)
        assert res[cap]["incumbent_steps"] > 3 and res[cap]["newcomer_ttft_ms"] is not None
        assert res[cap]["itl_max_ms"] >= res[cap]["itl_median_ms"]
    assert res[0]["prefill_steps"] == 3                        # 600 tokens at the 256-token chunk
    assert res[64]["prefill_steps"] == 10                      # 600 tokens at 64 per decode step


def test_apc_probe_reuses_the_shared_head():
    eng = _engine(checkpoints=4, checkpoint_pages=2)
    res = SP.apc(eng, [16 + (i * 13) % 480 for i in range(200)], [30, 31, 32, 33] * 8, gen=24)
    assert res["turn2_tokens"] == 200 + 24 + 32
    assert res["cached_tokens"] >= 192 and res["cold_cached_tokens"] == 0
    assert 0 < res["cached_fraction"] < 1
