"""Operator tooling on CPU: the boot checks' cross-rank environment agreement (gloo, world size 2), the
environment A/B driver (arms, interleaving, gates, verdict) with fake and real child commands, and the quality
probe's statistics (top-k union KL with the missing-mass floor, first divergence, run comparison)."""

import json
import math
import os
import sys

import pytest
import torch

from test_dist_cpu import _run


def _env_check(rank, world):
    import torch.distributed as dist
    from glm53.parallel import dist as D
    from glm53.utils import boot_checks
    os.environ["GLM53_PDL"] = "1"
    if rank == 1:
        os.environ["GLM53_OVERLAP"] = "1"
    D.init(backend="gloo", timeout_s=30)
    bad = boot_checks.check_env()
    os.environ.pop("GLM53_OVERLAP", None)
    good = boot_checks.check_env()
    dist.destroy_process_group()
    return bad, good


def test_boot_env_agreement_across_ranks():
    res = _run(_env_check, 2)
    for r in (0, 1):
        ok, payload = res[r]
        assert ok, payload
        bad, good = payload
        assert not bad["ok"] and bad["mismatch"] == {"GLM53_OVERLAP": [None, "1"]} and bad["ranks"] == 2
        assert good["ok"]


def test_boot_env_helpers():
    from glm53.utils import boot_checks as B
    env = {"GLM53_A": "1", "NCCL_ALGO": "Ring", "PATH": "/bin", "GLM53_TRACE": "/tmp/x"}
    assert B.switch_env(env) == {"GLM53_A": "1", "NCCL_ALGO": "Ring"}      # per-rank and unrelated names dropped
    assert B.env_mismatches([{"A": "1"}, {"A": "1"}]) == {}
    assert B.env_mismatches([{"A": "1"}, {"A": "2"}, {}]) == {"A": ["1", "2", None]}


def test_boot_run_without_gpu_reports_device():
    from glm53.utils import boot_checks as B
    if torch.cuda.is_available():
        pytest.skip("CPU-only expectation")
    rep = B.run()
    assert rep["env"]["ok"] and not rep["device"]["ok"] and not rep["ok"]
    with pytest.raises(RuntimeError, match="boot checks failed"):
        B.enforce(rep)


def test_arm_parse_and_refusals():
    from glm53.utils.arm_ab import parse_arm
    assert parse_arm("base") == ("base", {})
    assert parse_arm("w8:GLM53_PREFILL_W8A8=kda_in_proj,mla_o_proj,GLM53_PDL=0") == (
        "w8", {"GLM53_PREFILL_W8A8": "kda_in_proj,mla_o_proj", "GLM53_PDL": "0"})
    with pytest.raises(ValueError):
        parse_arm("x:API_KEY=1")                        # only GLM53_* / NCCL_* switches
    with pytest.raises(ValueError):
        parse_arm("x:GLM53_A=$(rm)")                     # no shell characters in values
    with pytest.raises(ValueError):
        parse_arm("Bad:GLM53_A=1")


def test_arm_ab_verdict_with_fake_runner():
    from glm53.utils import arm_ab
    calls = []
    speed = {"": 100.0, "fast": 110.0, "faster_bad": 130.0, "slow": 90.0}

    def runner(cmd, env, owned, timeout):
        calls.append((cmd, dict(env), set(owned)))
        v = speed[env.get("GLM53_X", "")]
        out = "noise\n" + ("proof: on\n" if env else "") + json.dumps({"value": v, "higher_is_better": True})
        if env.get("GLM53_X") == "faster_bad":
            out += "\nfallback used\n"
        return 0, out
    arms = [arm_ab.parse_arm(a) for a in ("base", "a:GLM53_X=fast", "b:GLM53_X=faster_bad", "c:GLM53_X=slow")]
    res = arm_ab.ab(arms, "bench", reps=2, proof=["proof: on"], never=["fallback used"], runner=runner)
    # interleaved order: base a b c base a b c
    assert [c[1].get("GLM53_X", "") for c in calls] == ["", "fast", "faster_bad", "slow"] * 2
    assert all(c[2] == {"GLM53_X"} for c in calls)
    assert res["arms"]["b"]["gates_failed"] == ["proof"]
    assert res["keep"] == "a" and res["keep_env"] == {"GLM53_X": "fast"}
    assert math.isclose(res["arms"]["a"]["gain_vs_base"], 0.1)
    res = arm_ab.ab(arms[:2], "bench", reps=1, min_gain=0.2, runner=runner)
    assert res["keep"] == "base"                          # 10 % is below the required gain


def test_arm_ab_quality_gate_and_lower_is_better():
    from glm53.utils import arm_ab

    def runner(cmd, env, owned, timeout):
        v = {"": 10.0, "1": 9.0, "2": 8.0}[env.get("GLM53_Y", "")]
        return 0, json.dumps({"value": v, "higher_is_better": False})
    arms = [("base", {}), ("one", {"GLM53_Y": "1"}), ("two", {"GLM53_Y": "2"})]
    quality = {"one": {"prefill": {"kl_mean": 0.001}, "decode_identical": 4, "decode_streams": 4},
               "two": {"prefill": {"kl_mean": 0.5}, "decode_identical": 4, "decode_streams": 4}}
    res = arm_ab.ab(arms, "bench", reps=1, probe="probe {arm}", compare=quality.get, max_kl=0.01, runner=runner)
    assert res["arms"]["two"]["gates_failed"] == ["kl"] and res["keep"] == "one"


def test_arm_ab_real_child_processes(tmp_path):
    """The default runner: child processes get the arm's switches and lose the owned ones from the parent."""
    from glm53.utils import arm_ab
    script = tmp_path / "b.py"
    script.write_text("import os, json\n"
                      "print(json.dumps({'value': float(os.environ.get('GLM53_ABTEST', '1')),"
                      " 'higher_is_better': True}))\n")
    os.environ["GLM53_ABTEST"] = "50"                     # owned by an arm: base must not see it
    try:
        res = arm_ab.ab([("base", {}), ("two", {"GLM53_ABTEST": "2"})], f"{sys.executable} {script}", reps=2)
    finally:
        os.environ.pop("GLM53_ABTEST")
    assert res["arms"]["base"]["values"] == [1.0, 1.0] and res["arms"]["two"]["values"] == [2.0, 2.0]
    assert res["keep"] == "two"


def test_quality_topk_kl():
    from glm53.utils.klh import kl_rows
    from glm53.utils.quality_probe import topk_kl, topk_logprobs
    g = torch.Generator().manual_seed(0)
    a, b = torch.randn(3, 32, generator=g), torch.randn(3, 32, generator=g)
    # with k = vocabulary the union KL is the exact KL
    pa, pb = topk_logprobs(a, 32), topk_logprobs(b, 32)
    exact = kl_rows(a, b)
    for i in range(3):
        assert math.isclose(topk_kl(pa[i], pb[i], 32), exact[i].item(), rel_tol=1e-9, abs_tol=1e-12)
        assert topk_kl(pa[i], pa[i], 32) == pytest.approx(0.0, abs=1e-12)
    # partial sets: finite, non-negative, zero for identical runs, and closer runs score lower
    qa, qb = topk_logprobs(a, 4), topk_logprobs(b, 4)
    assert all(0.0 <= topk_kl(x, y, 32) < math.inf for x, y in zip(qa, qb))
    assert all(topk_kl(x, x, 32) == pytest.approx(0.0, abs=1e-12) for x in qa)
    near = topk_logprobs(a + 0.01 * b, 4)
    assert all(topk_kl(x, y, 32) <= topk_kl(x, z, 32) + 1e-12 for x, y, z in zip(qa, near, qb))


def test_quality_compare_runs():
    from glm53.utils.quality_probe import compare_runs, first_divergence
    assert first_divergence([1, 2, 3], [1, 2, 3]) is None
    assert first_divergence([1, 2, 3], [1, 5, 3]) == 1
    assert first_divergence([1, 2], [1, 2, 3]) == 2
    lp = [[{"5": -0.1, "6": -2.5}, {"7": -0.3, "8": -1.5}]]
    A = {"completions": [[1, 2, 3], [4, 5]], "prompt_logprobs": lp, "vocab": 16}
    B = {"completions": [[1, 2, 3], [4, 9]], "prompt_logprobs": lp, "vocab": 16}
    r = compare_runs(A, B)
    assert r["decode_identical"] == 1 and r["first_divergence"] == [1]
    assert r["prefill"]["n"] == 2 and r["prefill"]["kl_max"] == pytest.approx(0.0, abs=1e-12)
    assert r["top1_agree"] == 1.0


def test_llm_boot_checks_refuse_to_start_without_a_b200(monkeypatch):
    """GLM53_BOOT_CHECKS=1: the engine runs the boot checks before touching a device and refuses to start when one
    fails (here: no CUDA device)."""
    if torch.cuda.is_available():
        pytest.skip("CPU-only expectation")
    from glm53.api.offline import LLM, LLMOptions
    monkeypatch.setenv("GLM53_BOOT_CHECKS", "1")
    with pytest.raises(RuntimeError, match="boot checks failed"):
        LLM(LLMOptions(model="tiny"))
