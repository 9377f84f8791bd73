"""Operational helpers of a serving process (the role of the reference's runtime helpers,
code/fork/glm53_runtime.py:285 profiler hook, :463 memory hygiene):

  install_profiler_signal(engine)   SIGUSR2 toggles a torch.profiler capture of the next N engine steps (CUDA
                                    activity), written as a Chrome trace next to GLM53_PROFILE_DIR
  memory_report()                   device memory of this process: allocated / reserved by the caching allocator,
                                    and the device's free / total
  trim_memory()                     return cached allocator blocks to the driver (after large prefills, before
                                    capturing more CUDA graphs)
"""

from __future__ import annotations

import os
import signal
import time

import torch


def memory_report(device=None) -> dict:
    if not torch.cuda.is_available():
        return {"cuda": False}
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    free, total = torch.cuda.mem_get_info(dev)
    return {"allocated_gib": torch.cuda.memory_allocated(dev) / 2 ** 30,
            "reserved_gib": torch.cuda.memory_reserved(dev) / 2 ** 30,
            "device_free_gib": free / 2 ** 30, "device_total_gib": total / 2 ** 30}


def trim_memory() -> None:
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


class _StepProfiler:
    def __init__(self, engine, steps: int, out_dir: str):
        self.engine, self.steps, self.out_dir = engine, steps, out_dir
        self.armed = False
        self.left = 0
        self.prof = None
        step = engine.step

        def wrapped():
            if self.armed and self.prof is None:
                from torch.profiler import ProfilerActivity, profile
                acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
                self.prof = profile(activities=acts)
                self.prof.__enter__()
                self.left = self.steps
            out = step()
            if self.prof is not None:
                self.left -= 1
                if self.left <= 0:
                    if torch.cuda.is_available():
                        torch.cuda.synchronize()
                    self.prof.__exit__(None, None, None)
                    os.makedirs(self.out_dir, exist_ok=True)
                    path = os.path.join(self.out_dir, f"steps-{int(time.time())}-pid{os.getpid()}.json")
                    self.prof.export_chrome_trace(path)
                    self.last_path = path
                    self.prof = None
                    self.armed = False
            return out
        engine.step = wrapped

    def arm(self, *_):
        self.armed = True


def install_profiler_signal(engine, steps: int = 8, out_dir: str | None = None, sig=signal.SIGUSR2):
    """After ``kill -USR2 <pid>`` the next ``steps`` engine steps are profiled; returns the controller (its
    ``arm()`` does the same without a signal)."""
    ctl = _StepProfiler(engine, steps, out_dir or os.environ.get("GLM53_PROFILE_DIR", "profiles_runtime"))
    try:
        signal.signal(sig, ctl.arm)
    except ValueError:                   # not the main thread: arming by signal is unavailable, arm() still works
        pass
    return ctl
