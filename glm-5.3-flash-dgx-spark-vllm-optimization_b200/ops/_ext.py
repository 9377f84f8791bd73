"""Build and load the in-tree CUDA extension (``glm53_C``) for sm_100a.

The extension is compiled with nvcc for ``-gencode arch=compute_100a,code=sm_100a`` only (no other architecture)
into ``<package>/_build/``, next to the sources, so the built ``.so`` travels with the source tree.  ``load()``
imports a built library directly (no rebuild check) and builds it when it is missing; ``build()`` always runs the
(incremental, ninja) build.  On a machine with a CUDA device the extension is mandatory: ``require()`` raises if it
cannot be loaded, so no op silently falls back to PyTorch.

``GLM53_BOUNDS=1`` selects the bounds-checked debug build instead: the same sources compiled with
``-DG53_BOUNDS=1`` into ``glm53_C_bounds`` under ``<package>/_build_bounds/``.  Its kernels check every index
they read from device data (token ids, cache slots, state slots, expert ids, token rows of the MoE pairs) against
the tensor it indexes, skip the access when it is out of range and record the first failure per compilation unit;
``bounds_status()`` / ``bounds_reset()`` of the module read and clear the records.
"""

from __future__ import annotations

import glob
import importlib.util
import os
import sys
import threading

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(_PKG, "csrc")
BOUNDS = os.environ.get("GLM53_BOUNDS", "0") == "1"
BUILD_DIR = os.path.join(_PKG, "_build_bounds" if BOUNDS else "_build")
NAME = "glm53_C_bounds" if BOUNDS else "glm53_C"
ARCH_FLAGS = ["-gencode=arch=compute_100a,code=sm_100a"]
_DEFS = ["-DG53_BOUNDS=1"] if BOUNDS else []
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v"] + _DEFS

_lock = threading.Lock()
_mod = None


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))


def so_path() -> str:
    return os.path.join(BUILD_DIR, NAME + ".so")


def stale() -> bool:
    """True when a source or header is newer than the built library."""
    so = so_path()
    if not os.path.exists(so):
        return True
    t = os.path.getmtime(so)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    return any(os.path.getmtime(f) > t for f in deps)


def build(verbose: bool = False):
    """Compile every CUDA source for sm_100a (incremental) and return the loaded module."""
    global _mod
    import torch.utils.cpp_extension as ce
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))
    # the -gencode flags in extra_cuda_cflags replace torch's own arch list
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    with _lock:
        _mod = ce.load(name=NAME, sources=sources(), extra_cuda_cflags=NVCC_FLAGS,
                       extra_cflags=["-O3", "-std=c++17"] + _DEFS, build_directory=BUILD_DIR, verbose=verbose,
                       with_cuda=True)
    return _mod


def _import_so(path: str):
    import torch  # noqa: F401  (the extension links against torch's libraries)
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod


def load(build_if_missing: bool = True):
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        if os.path.exists(so_path()) and not stale():
            _mod = _import_so(so_path())
            return _mod
    if build_if_missing:
        return build()
    return None


def require():
    """The extension, or an exception: kernels never fall back to eager PyTorch on a GPU machine."""
    try:
        mod = load()
    except Exception as e:  # pragma: no cover - exercised only when the build is broken
        raise RuntimeError(f"glm53 CUDA extension could not be loaded: {e}") from e
    if mod is None:
        raise RuntimeError("glm53 CUDA extension is not built (run __graft_entry__.build())")
    return mod
