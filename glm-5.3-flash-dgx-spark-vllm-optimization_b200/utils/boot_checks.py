"""Per-rank boot assertions of a serving process (the role of the reference's boot-log checks,
code/kit/tools/boot_checks.sh:1-30, which grep every rank's log for the install / self-test / serving lines and
require the head's and the worker's environment to match).  Here the checks run in-process, before the first
request, and return a structured report instead of log lines:

  device      the GPU is an sm_100 part; SM count, memory
  extension   the in-tree sm_100a extension is built and loaded from this tree (no PyTorch fallback exists)
  selftest    a few kernels against fp32 PyTorch on tiny inputs (fp8 GEMV, bf16 GEMV) -- the self-test line
  env         every rank sees the same GLM53_* / NCCL_* switches (a mismatch between ranks changes which kernels
              run on each rank, the reference's head == worker rule); gathered over the default process group

    python -m glm53.utils.boot_checks            # one process
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m glm53.utils.boot_checks

`LLM(...)` runs them at boot when GLM53_BOOT_CHECKS=1 and raises on a failed check.
"""

from __future__ import annotations

import json
import math
import os

import torch

ENV_PREFIXES = ("GLM53_", "NCCL_")
# per-process values that legitimately differ between ranks
ENV_PER_RANK = {"GLM53_TRACE", "GLM53_PROFILE_DIR", "NCCL_DEBUG_FILE"}


def switch_env(environ=None) -> dict:
    environ = os.environ if environ is None else environ
    return {k: v for k, v in sorted(environ.items())
            if k.startswith(ENV_PREFIXES) and k not in ENV_PER_RANK}


def env_mismatches(envs: list[dict]) -> dict:
    """key -> [value on rank 0, value on rank 1, ...] for every switch whose value is not the same on all ranks
    (None where a rank does not set it)."""
    keys = sorted(set().union(*[e.keys() for e in envs])) if envs else []
    out = {}
    for k in keys:
        vals = [e.get(k) for e in envs]
        if any(v != vals[0] for v in vals):
            out[k] = vals
    return out


def check_env(group=None) -> dict:
    import torch.distributed as dist
    mine = switch_env()
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return {"ok": True, "ranks": 1, "switches": len(mine)}
    envs = [None] * dist.get_world_size(group)
    dist.all_gather_object(envs, mine, group=group)
    bad = env_mismatches(envs)
    return {"ok": not bad, "ranks": len(envs), "switches": len(mine), "mismatch": bad}


def check_device() -> dict:
    if not torch.cuda.is_available():
        return {"ok": False, "why": "no CUDA device"}
    i = torch.cuda.current_device()
    p = torch.cuda.get_device_properties(i)
    cap = (p.major, p.minor)
    return {"ok": cap == (10, 0), "name": p.name, "capability": f"{cap[0]}.{cap[1]}",
            "sms": p.multi_processor_count, "memory_gib": round(p.total_memory / 2 ** 30, 1)}


def check_extension() -> dict:
    from ..ops import _ext
    try:
        mod = _ext.require()
    except Exception as e:                                          # noqa: BLE001 -- reported, then raised by run()
        return {"ok": False, "why": f"{type(e).__name__}: {e}"}
    path = os.path.realpath(getattr(mod, "__file__", "") or "")
    tree = os.path.realpath(_ext.BUILD_DIR)
    return {"ok": path.startswith(tree), "so": path}


def check_selftest() -> dict:
    """fp8 and bf16 GEMV against fp32 PyTorch on tiny shapes (one launch each)."""
    from ..models.weights import quantize_fp8_rows
    from ..ops import kernels as K
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(7)
    M, N, Kd = 4, 256, 512
    w = quantize_fp8_rows(torch.randn(N, Kd, device=dev, generator=g) / math.sqrt(Kd))
    x = torch.randn(M, Kd, device=dev, generator=g).to(torch.bfloat16)
    ref = x.float() @ w.dequant().t()
    y = torch.empty(M, N, dtype=torch.float32, device=dev)
    K.C().gemv(x, w.w, w.s, y, K.GEMV_F32, 0.0)
    wb = (torch.randn(N, Kd, device=dev, generator=g) / math.sqrt(Kd)).to(torch.bfloat16)
    yb = torch.empty(M, N, dtype=torch.float32, device=dev)
    K.linear_bf16(x, wb, yb)
    refb = x.float() @ wb.float().t()
    torch.cuda.synchronize()
    e8 = (y - ref).abs().max().item()
    eb = (yb - refb).abs().max().item()
    return {"ok": e8 < 2e-3 and eb < 2e-3, "gemv_fp8_max_err": e8, "gemv_bf16_max_err": eb}


def run(group=None, selftest: bool = True) -> dict:
    """All checks of this rank; report["ok"] is the conjunction.  The env check is collective: every rank of the
    group must call run() (it is the only collective step and comes first, so a rank whose device check fails
    still takes part in it)."""
    rep = {"env": check_env(group)}
    from .switches import check as check_switches
    rep["switches"] = check_switches()
    rep["device"] = check_device()
    if rep["device"]["ok"]:
        rep["extension"] = check_extension()
        if selftest and rep["extension"]["ok"]:
            rep["selftest"] = check_selftest()
    rep["ok"] = all(v["ok"] for v in rep.values() if isinstance(v, dict))
    return rep


def enforce(report: dict) -> None:
    if not report["ok"]:
        failed = {k: v for k, v in report.items() if isinstance(v, dict) and not v["ok"]}
        raise RuntimeError(f"boot checks failed: {json.dumps(failed)}")


def main(argv=None):
    from ..parallel import dist as D
    rank, _, world = D.init()
    rep = run()
    rep["rank"] = rank
    print(json.dumps(rep), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
