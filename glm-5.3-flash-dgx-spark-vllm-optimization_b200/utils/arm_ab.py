"""Environment-switch A/B driver (the role of the reference's production A/B, code/kit/tools/arm_env_ab.sh:1-45: arms
of operator switches, a measurement per arm, gates, keep the best).  One arm is a named set of GLM53_* / NCCL_*
assignments; "base" (no assignments) always runs.  For every repetition the arms run in turn (base, a, b, base, a,
b, ...), so a drift of the machine hits every arm alike.  Each run is a child process with the arm's environment:

  measure  the benchmark command (default: bench.py on one GPU); its last JSON line gives the metric
           ("value", and "higher_is_better")
  proof    fixed strings that must appear in a non-base arm's output (the switch really took effect), and strings
           that must not (a refusal or fallback line)
  probe    optional quality command run once per arm after its measurements, with {arm} in the command replaced by
           the arm name (e.g. the quality probe writing <arm>.json); a non-base arm whose probe compared against
           base's exceeds --max-kl, or whose decode diverges when --require-identical is set, is rejected

The verdict keeps the arm with the best median among the arms that passed every gate and beat base by --min-gain
(relative); otherwise base.

    python -m glm53.utils.arm_ab --arm pdl_off:GLM53_PDL=0 --arm overlap:GLM53_OVERLAP=1 --reps 3 \
        --probe "python -m glm53.utils.quality_probe run --out {arm}.json"
"""

from __future__ import annotations

import argparse
import json
import os
import re
import shlex
import statistics
import subprocess
import sys

ALLOWED = re.compile(r"^(GLM53_[A-Z0-9_]+|NCCL_[A-Z0-9_]+)$")
VALUE = re.compile(r"^[A-Za-z0-9_.,:/+-]*$")
NAME = re.compile(r"^[a-z0-9_]+$")


def parse_arm(spec: str) -> tuple[str, dict]:
    """'name:K=V,K2=V2' (or 'name' for no assignments) -> (name, {K: V}); names and values are checked."""
    name, _, rest = spec.partition(":")
    if not NAME.match(name):
        raise ValueError(f"arm name {name!r}: lower-case letters, digits and _ only")
    env = {}
    for kv in filter(None, re.split(r"[ ,](?=[A-Z])", rest)):
        k, sep, v = kv.partition("=")
        if not sep or not ALLOWED.match(k):
            raise ValueError(f"arm {name}: {kv!r} is not a GLM53_*/NCCL_* assignment")
        if not VALUE.match(v):
            raise ValueError(f"arm {name}: value of {k} has characters outside [A-Za-z0-9_.,:/+-]")
        env[k] = v
    return name, env


def last_json(text: str) -> dict | None:
    for line in reversed(text.splitlines()):
        line = line.strip()
        if line.startswith("{") and line.endswith("}"):
            try:
                return json.loads(line)
            except json.JSONDecodeError:
                continue
    return None


def run_cmd(cmd: str, env_add: dict, owned: set, timeout: float) -> tuple[int, str]:
    """The command with this process's environment minus every switch an arm owns, plus this arm's values."""
    env = {k: v for k, v in os.environ.items() if k not in owned}
    env.update(env_add)
    p = subprocess.run(shlex.split(cmd), env=env, capture_output=True, text=True, timeout=timeout)
    return p.returncode, p.stdout + p.stderr


def ab(arms: list[tuple[str, dict]], cmd: str, reps: int = 3, proof: list[str] = (), never: list[str] = (),
       probe: str | None = None, compare=None, max_kl: float | None = None, require_identical: bool = False,
       min_gain: float = 0.0, timeout: float = 1800.0, runner=run_cmd) -> dict:
    """Run the A/B; returns per-arm values, gates and the verdict.  `compare(arm_name)` gives the quality
    statistics of that arm's probe output against base's (the quality probe's compare of the two saved runs)."""
    if not arms or arms[0][0] != "base":
        arms = [("base", {})] + [a for a in arms if a[0] != "base"]
    res = {name: {"env": env, "values": [], "failures": [], "proof_ok": True} for name, env in arms}
    owned = set().union(*[set(env) for _, env in arms])
    hib = True
    for _ in range(reps):
        for name, env in arms:
            code, out = runner(cmd, env, owned, timeout)
            js = last_json(out)
            if code != 0 or js is None or "value" not in js:
                res[name]["failures"].append(code)
                continue
            hib = bool(js.get("higher_is_better", True))
            res[name]["values"].append(float(js["value"]))
            if name != "base":
                ok = all(s in out for s in proof) and not any(s in out for s in never)
                res[name]["proof_ok"] = res[name]["proof_ok"] and ok
    probes = {}
    if probe:
        for name, env in arms:
            code, out = runner(probe.replace("{arm}", name), env, owned, timeout)
            probes[name] = {"code": code, "out": last_json(out)}
            res[name]["probe_code"] = code
    for name, _ in arms:
        r = res[name]
        r["median"] = statistics.median(r["values"]) if r["values"] else None
        gates = []
        if r["failures"]:
            gates.append("run failed")
        if not r["proof_ok"]:
            gates.append("proof")
        if probe and name != "base":
            if probes[name]["code"] != 0:
                gates.append("probe failed")
            elif compare is not None:
                q = compare(name)
                r["quality"] = q
                kl = (q.get("prefill") or {}).get("kl_mean")
                if max_kl is not None and kl is not None and kl > max_kl:
                    gates.append("kl")
                if require_identical and q.get("decode_identical") != q.get("decode_streams"):
                    gates.append("decode diverged")
        r["gates_failed"] = gates
    base = res["base"]["median"]
    best, best_v = "base", base
    for name, _ in arms[1:]:
        r = res[name]
        v = r["median"]
        if r["gates_failed"] or v is None or base is None:
            continue
        gain = (v - base) / abs(base) if hib else (base - v) / abs(base)
        r["gain_vs_base"] = gain
        better = (v > best_v) if hib else (v < best_v)
        if gain >= min_gain and better:
            best, best_v = name, v
    return {"arms": res, "higher_is_better": hib, "keep": best, "keep_env": dict(arms)[best] if best else {}}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--arm", action="append", default=[], help="name:GLM53_X=1,GLM53_Y=2 (repeatable)")
    ap.add_argument("--cmd", default=f"{sys.executable} bench.py --gpus 1 --steps 20 --warmup 3")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--proof", action="append", default=[])
    ap.add_argument("--never", action="append", default=[])
    ap.add_argument("--probe", default=None, help="quality command, {arm} -> arm name")
    ap.add_argument("--probe-out", default="{arm}.json", help="file the probe writes, {arm} -> arm name")
    ap.add_argument("--max-kl", type=float, default=None)
    ap.add_argument("--require-identical", action="store_true")
    ap.add_argument("--min-gain", type=float, default=0.0)
    ap.add_argument("--timeout", type=float, default=1800.0)
    args = ap.parse_args(argv)
    arms = [parse_arm("base")] + [parse_arm(a) for a in args.arm]
    compare = None
    if args.probe:
        from .quality_probe import compare_runs

        def compare(name):
            with open(args.probe_out.replace("{arm}", "base")) as fa, \
                 open(args.probe_out.replace("{arm}", name)) as fb:
                return compare_runs(json.load(fa), json.load(fb))
    out = ab(arms, args.cmd, args.reps, args.proof, args.never, args.probe, compare, args.max_kl,
             args.require_identical, args.min_gain, args.timeout)
    print(json.dumps(out), flush=True)
    return out


if __name__ == "__main__":
    main()
