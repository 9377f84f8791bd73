"""Environment switches: every GLM53_* name the sources read is in the table, defaults validate, typos are reported
with the closest name, malformed values are refused (and stop LLM before it touches a device)."""

import pathlib
import re

import pytest

from glm53.utils import switches as S

PKG = pathlib.Path(__file__).resolve().parents[1] / "glm-5.3-flash-dgx-spark-vllm-optimization_b200"
NOT_SWITCHES = {"GLM53_X", "GLM53_Y", "GLM53_DENSE_W8A8_ONLY"}   # a help-text example; the reference's name


def test_every_switch_in_the_sources_is_registered():
    names = set()
    for f in list(PKG.rglob("*.py")) + list(PKG.rglob("*.cu")) + list(PKG.rglob("*.cpp")) + list(PKG.rglob("*.cuh")):
        names |= set(re.findall(r"GLM53_[A-Z0-9_]+", f.read_text(errors="ignore")))
    assert names - NOT_SWITCHES - set(S.SWITCHES) == set()
    assert set(S.SWITCHES) - names == set()                    # no stale entries


def test_defaults_validate_and_bad_values_are_reported():
    assert S.check({k: v.default for k, v in S.SWITCHES.items()})["ok"]
    rep = S.check({"GLM53_PDL": "2", "GLM53_PDLL": "0", "GLM53_L2_PREFETCH_MB": "-1",
                   "GLM53_PREFILL_W8A8": "kda_in_proj,bogus", "GLM53_BULK_GEMV_MIN": "4M", "PATH": "/bin"})
    assert not rep["ok"]
    assert rep["unknown"] == {"GLM53_PDLL": "GLM53_PDL"}
    assert set(rep["malformed"]) == {"GLM53_PDL", "GLM53_L2_PREFETCH_MB", "GLM53_PREFILL_W8A8",
                                     "GLM53_BULK_GEMV_MIN"}
    assert S.check({"GLM53_PREFILL_W8A8": "none"})["ok"] and S.check({"GLM53_PREFILL_W8A8": "ALL"})["ok"]


def test_llm_refuses_malformed_switches(monkeypatch):
    from glm53.api.offline import LLM, LLMOptions
    monkeypatch.setenv("GLM53_FUSED_TP", "yes")
    with pytest.raises(ValueError, match="GLM53_FUSED_TP"):
        LLM(LLMOptions(model="tiny"))


def test_unknown_switch_warns():
    with pytest.warns(UserWarning, match="did you mean GLM53_OVERLAP"):
        S.enforce({"GLM53_OVERLAPP": "1"})
