"""The sampled-decoding bench's statistics on CPU: the engine's window counters (windows, accepted drafts, per-position
acceptance) turned into accepted tokens per step, per-position acceptance and draft tokens per step, per request, with
the fake backend (greedy speculative decoding; its drafter errs on every third position)."""

import json

import pytest

from glm53.engine.llm import EngineConfig, LLMEngine, SamplingParams
from glm53.utils import bench_sampled as BS
from tests.fake_backend import FakeBackend


def _engine(**kw):
    cfg = EngineConfig(**{"max_seqs": 1, "page_size": 16, "num_pages": 64, "max_model_len": 512,
                          "prefill_chunk": 64, "cuda_graphs": False, "k_fixed": 4, **kw})
    return LLMEngine(FakeBackend(max_seqs=1, checkpoints=0), cfg)


def test_window_stats_arithmetic():
    m0 = {"spec_windows": 10, "steps": 12, "spec_accepted": 20, "spec_drafts": 40,
          "spec_accepted_per_pos": [8, 6, 4, 2] + [0] * 12}
    m1 = {"spec_windows": 20, "steps": 22, "spec_accepted": 45, "spec_drafts": 80,
          "spec_accepted_per_pos": [18, 14, 9, 4] + [0] * 12}
    st = BS.window_stats(m0, m1, tokens=35, seconds=0.5)
    assert st["windows"] == 10 and st["steps"] == 10
    assert st["accepted_per_step"] == pytest.approx(3.5)
    assert st["draft_tokens_per_step"] == pytest.approx(4.0)
    assert st["acceptance_per_position"][:4] == pytest.approx([1.0, 0.8, 0.5, 0.2])
    assert st["tok_s"] == pytest.approx(70.0) and st["ms_per_step"] == pytest.approx(50.0)
    assert "accepted_per_step" not in BS.window_stats(m0, m0, 0, 0.0)


def test_run_reports_per_request_window_statistics():
    eng = _engine()
    prompts = [[3, 5, 7, 9] * 10, [11, 2, 4] * 12]
    rows = BS.run(eng, prompts, lambda i: SamplingParams(max_tokens=40, seed=100 + i, ignore_eos=True))
    assert len(rows) == 2
    for r in rows:
        assert r["windows"] > 0 and r["tokens"] > 0
        # every window emits its accepted drafts plus one token; the last window may be cut by max_tokens
        assert r["tokens"] <= r["windows"] * r["accepted_per_step"] + 1e-9
        assert 1.0 <= r["accepted_per_step"] <= 5.0
        assert r["draft_tokens_per_step"] == pytest.approx(4.0)
        pos = r["acceptance_per_position"]
        assert all(a >= b for a, b in zip(pos, pos[1:]))        # accepting position i needs every earlier one
        assert sum(pos) == pytest.approx(r["accepted_per_step"] - 1.0)
    s = BS.summary(rows)
    assert s["accepted_per_step"] == pytest.approx(sum(r["accepted_per_step"] for r in rows) / 2)


def test_compare_reads_two_runs(tmp_path, capsys):
    a, b = tmp_path / "a.json", tmp_path / "b.json"
    a.write_text(json.dumps({"summary": {"accepted_per_step": 3.0}}))
    b.write_text(json.dumps({"summary": {"accepted_per_step": 3.4}}))
    res = BS.main(["--compare", str(a), str(b)])
    assert res["summary_a"]["accepted_per_step"] == 3.0 and res["summary_b"]["accepted_per_step"] == 3.4
    assert "3.4" in capsys.readouterr().out
