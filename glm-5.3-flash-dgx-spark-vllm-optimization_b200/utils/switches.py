"""The engine's environment switches in one table, and their validation. The reference's launcher refuses to start on
a malformed numeric setting (code/kit/launcher/start.sh:853, ``validate_numeric_config``) and checks its env files
(code/kit/tools/check_config.sh); here every ``GLM53_*`` variable of the process is checked against this table:

  unknown     a GLM53_* name the engine does not read (a typo would otherwise be ignored silently); the closest known
              name is suggested
  malformed   a value the reader would misread (a boolean other than 0 / 1, a negative size, an unknown projection)

``LLM`` refuses to start on a malformed value and warns about unknown names; the boot checks report both.
"""

from __future__ import annotations

import difflib
import os
from dataclasses import dataclass

W8A8_PROJECTIONS = ("kda_in_proj", "mla_o_proj")


@dataclass(frozen=True)
class Switch:
    kind: str          # "bool" | "int" | "float" | "path" | "projections"
    default: str
    help: str


SWITCHES: dict[str, Switch] = {
    "GLM53_PDL": Switch("bool", "1", "programmatic dependent launches on the decode kernel chain"),
    "GLM53_OVERLAP": Switch("bool", "1", "second stream for independent work inside a step"),
    "GLM53_KDA_FUSED": Switch("bool", "1", "decode windows run the KDA block tail as one kernel"),
    "GLM53_HC_FUSED": Switch("bool", "1", "decode windows run mHC post + pre as one cluster kernel"),
    "GLM53_TC_HC": Switch("bool", "1", "prefill-sized mHC launches use the tensor-core partial pass"),
    "GLM53_TC_MLA": Switch("bool", "1", "tensor-core sparse MLA kernel where its shape applies"),
    "GLM53_TC_DSA": Switch("bool", "1", "tcgen05 DSA indexer logits"),
    "GLM53_TCGEN05_GEMM": Switch("bool", "1", "large-M projections on the tcgen05 GEMM"),
    "GLM53_BULK_GEMV": Switch("bool", "1", "large fp8 projections on the bulk-copy GEMV"),
    "GLM53_BULK_GEMV_MIN": Switch("int", str(4 << 20), "weight bytes from which the bulk-copy GEMV is used"),
    "GLM53_FUSED_TP": Switch("bool", "1", "decode windows reduce tensor-parallel partials inside the kernels"),
    "GLM53_FUSED_TP_PREFILL": Switch("bool", "0", "prefill chunks push partials from the GEMM epilogue"),
    "GLM53_SP": Switch("bool", "1", "sequence-parallel prefill: mHC on each rank's rows, all-gather / reduce-scatter"),
    "GLM53_SP_MIN_ROWS": Switch("int", "256", "rows of a prefill chunk from which sequence parallelism is used"),
    "GLM53_MOE_DECODE_SPLIT": Switch("int", "0", "decode MoE gate/up: K split over a cluster (1, 2, 4, 8; 0 = "
                                                "chosen from the grid size), for tuning"),
    "GLM53_SP_FP8AG": Switch("bool", "1", "sequence-parallel prefill all-gathers the KDA input rows as e4m3 codes "
                                          "when that projection runs W8A8"),
    "GLM53_SP_MLA": Switch("bool", "1", "sequence-parallel prefill runs the MLA attention of each rank's rows over "
                                        "all heads (keeps the full-head MLA projections on every rank)"),
    "GLM53_BOUNDS": Switch("bool", "0", "load the bounds-checked debug build (glm53_C_bounds): device indices "
                                        "checked against their tensors, guard bands around runtime scratch"),
    "GLM53_L2_PREFETCH": Switch("bool", "0", "routed-expert CTAs prefetch the next layer's weights into L2"),
    "GLM53_L2_PREFETCH_MB": Switch("float", "32", "L2 prefetch budget in MiB"),
    "GLM53_PREFILL_W8A8": Switch("projections", ",".join(W8A8_PROJECTIONS),
                                 "prefill projections with e4m3 activations (list, all or none)"),
    "GLM53_BOOT_CHECKS": Switch("bool", "0", "run the boot checks before the engine starts"),
    "GLM53_TRACE": Switch("path", "", "write per-step trace records to this path"),
    "GLM53_PROFILE_DIR": Switch("path", "profiles_runtime", "directory of the SIGUSR2 step profiles"),
}


def _malformed(sw: Switch, value: str) -> str | None:
    v = value.strip()
    if sw.kind == "bool":
        return None if v in ("0", "1") else "expected 0 or 1"
    if sw.kind in ("int", "float"):
        try:
            x = int(v) if sw.kind == "int" else float(v)
        except ValueError:
            return f"expected a non-negative {sw.kind}"
        return None if x >= 0 else f"expected a non-negative {sw.kind}"
    if sw.kind == "projections":
        if v.lower() in ("", "0", "1", "all", "none"):
            return None
        bad = [p for p in (s.strip() for s in v.lower().split(",")) if p not in W8A8_PROJECTIONS]
        return f"unknown projection(s) {bad}; known: {list(W8A8_PROJECTIONS)}" if bad else None
    return None


def check(env=None) -> dict:
    env = os.environ if env is None else env
    unknown, malformed = {}, {}
    for name, value in env.items():
        if not name.startswith("GLM53_"):
            continue
        sw = SWITCHES.get(name)
        if sw is None:
            close = difflib.get_close_matches(name, SWITCHES, n=1)
            unknown[name] = close[0] if close else None
            continue
        why = _malformed(sw, value)
        if why:
            malformed[name] = f"{value!r}: {why}"
    return {"ok": not unknown and not malformed, "unknown": unknown, "malformed": malformed}


def enforce(env=None) -> dict:
    """Raise on malformed values; warn about unknown names. Returns the report."""
    rep = check(env)
    if rep["malformed"]:
        raise ValueError(f"malformed GLM53_* switches: {rep['malformed']}")
    if rep["unknown"]:
        import warnings
        hints = {k: (f"did you mean {v}?" if v else "not read by the engine") for k, v in rep["unknown"].items()}
        warnings.warn(f"unknown GLM53_* switches: {hints}", stacklevel=2)
    return rep


def table() -> list[dict]:
    return [{"name": k, "kind": v.kind, "default": v.default, "help": v.help} for k, v in SWITCHES.items()]


if __name__ == "__main__":
    import json
    print(json.dumps({"switches": table(), "check": check()}, indent=1))
