"""Operator tools on the GPU with the tiny proxy: the boot checks pass (sm_100 device, in-tree extension, kernel
self-test), the decode-vs-prefill probe finds the decode kernels and the prefill kernels in agreement, and the
concurrency probe finds speculative greedy decoding token-identical to plain greedy decoding."""

import pytest

pytestmark = pytest.mark.gpu


def test_boot_checks_pass():
    from glm53.utils import boot_checks
    rep = boot_checks.run()
    assert rep["ok"], rep
    assert rep["device"]["capability"] == "10.0" and rep["extension"]["so"].endswith(".so")
    assert rep["selftest"]["gemv_fp8_max_err"] < 2e-3


def test_quality_probe_decode_vs_prefill():
    from glm53.utils import quality_probe as Q
    res = Q.main(["dvp", "--model", "tiny", "--len", "256", "--prompts", "2", "--window", "8", "--chunk", "128"])
    assert res["top1_agree"] >= 0.9, res
    for b in res["buckets"].values():
        assert b["kl_mean"] < 1e-2, res


def test_quality_probe_concurrency():
    from glm53.utils import quality_probe as Q
    res = Q.main(["conc", "--model", "tiny", "--len", "200", "--streams", "3", "--gen", "32"])
    assert res["spec_identical"] == 3, res
    assert res["conc_token_agree"] >= 0.5, res
