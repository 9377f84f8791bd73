"""Decode-step tracing (the role of the reference's dectrace, code/fork/glm53_dectrace.py:97, :490): per engine step
the host timestamps of the step and of each backend call, and every collective of the communicator timed on the
device with CUDA events, so per-rank host gaps and rank skew (one rank arriving late to an all-reduce) can be read
from the records.  Records are JSON lines, one per step and rank:

    {"rank": r, "step": n, "t0": unix_s, "host_ms": ..., "phases_ms": {"backend.verify": ...},
     "collectives": [{"op": "all_reduce", "bytes": b, "device_ms": t}, ...]}

Enable with GLM53_TRACE=<path> (each rank appends to <path>.rank<r>) or ``StepTracer(path).attach(engine, comm)``.
Device times are resolved once per step (one synchronize at the end of the traced step), so tracing perturbs the
timing it records only by that synchronize.
"""

from __future__ import annotations

import json
import os
import time

import torch


class StepTracer:
    def __init__(self, path: str, rank: int = 0):
        self.path = f"{path}.rank{rank}"
        self.rank = rank
        self.step = 0
        self._coll: list = []
        self._phase: dict = {}
        self._f = open(self.path, "a")

    # ------------------------------------------------------------------------------------------------ wiring
    def attach(self, engine, comm=None):
        """Wrap engine.step, the backend's calls and the communicator's collectives."""
        step = engine.step

        def traced_step():
            t0 = time.time()
            h0 = time.perf_counter()
            out = step()
            if torch.cuda.is_available():
                torch.cuda.synchronize()
            self.emit(t0, (time.perf_counter() - h0) * 1e3)
            return out
        engine.step = traced_step
        b = engine.b
        for name in ("prefill", "verify", "argmax", "commit", "draft"):
            if hasattr(b, name):
                setattr(b, name, self._wrap_phase(getattr(b, name), "backend." + name))
        if comm is not None:
            for op in ("all_reduce", "all_gather"):
                if hasattr(comm, op):
                    setattr(comm, op, self._wrap_coll(getattr(comm, op), op))
        return self

    def _wrap_phase(self, fn, label):
        def timed(*a, **k):
            h0 = time.perf_counter()
            try:
                return fn(*a, **k)
            finally:
                self._phase[label] = self._phase.get(label, 0.0) + (time.perf_counter() - h0) * 1e3
        return timed

    def _wrap_coll(self, fn, op):
        def timed(*a, **k):
            t = a[-1] if a else None
            nbytes = t.numel() * t.element_size() if isinstance(t, torch.Tensor) else 0
            if torch.cuda.is_available():
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                out = fn(*a, **k)
                e1.record()
                self._coll.append((op, nbytes, e0, e1))
                return out
            h0 = time.perf_counter()
            out = fn(*a, **k)
            self._coll.append((op, nbytes, (time.perf_counter() - h0) * 1e3, None))
            return out
        return timed

    # ------------------------------------------------------------------------------------------------ records
    def emit(self, t0: float, host_ms: float) -> None:
        colls = []
        for op, nbytes, e0, e1 in self._coll:
            ms = e0.elapsed_time(e1) if e1 is not None else e0
            colls.append({"op": op, "bytes": nbytes, "device_ms": ms})
        rec = {"rank": self.rank, "step": self.step, "t0": t0, "host_ms": host_ms,
               "phases_ms": dict(self._phase), "collectives": colls}
        self._f.write(json.dumps(rec) + "\n")
        self._f.flush()
        self._coll.clear()
        self._phase.clear()
        self.step += 1

    def close(self):
        self._f.close()


def maybe_attach(engine, comm=None, rank: int = 0):
    """Attach a tracer when GLM53_TRACE is set; returns it (or None)."""
    path = os.environ.get("GLM53_TRACE")
    if not path:
        return None
    return StepTracer(path, rank).attach(engine, comm)


def rank_skew(paths: list[str]) -> list[dict]:
    """Per step across ranks: host start skew and the spread of each collective's device time (the late rank's
    peers wait inside the collective, so its device time is the shortest)."""
    recs = []
    for p in paths:
        with open(p) as f:
            recs.append([json.loads(l) for l in f if l.strip()])
    out = []
    for step in range(min(len(r) for r in recs)):
        rows = [r[step] for r in recs]
        t0 = [x["t0"] for x in rows]
        n = min(len(x["collectives"]) for x in rows)
        spread = [max(x["collectives"][i]["device_ms"] for x in rows) - min(x["collectives"][i]["device_ms"]
                                                                            for x in rows) for i in range(n)]
        out.append({"step": step, "start_skew_ms": (max(t0) - min(t0)) * 1e3,
                    "max_collective_spread_ms": max(spread) if spread else 0.0})
    return out
