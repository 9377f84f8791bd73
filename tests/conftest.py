import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")
    config.addinivalue_line("markers", "w8a8: runs with the default prefill W8A8 policy (others: exact W8A16)")


@pytest.fixture(autouse=True)
def _exact_prefill_projections(request, monkeypatch):
    """Numerics tests compare against the fp32 oracle and across prefill / decode paths, so large-M projections run
    in exact W8A16 unless a test is marked `w8a8` (the default policy quantises two projections' activations)."""
    if request.node.get_closest_marker("w8a8"):
        yield
        return
    try:
        from glm53.ops import kernels as K
    except Exception:  # pragma: no cover - the package imports on every supported host
        yield
        return
    monkeypatch.setattr(K, "W8A8_PROJ", set())
    monkeypatch.setattr(K, "PREFILL_W8A8", False)
    yield


@pytest.fixture(autouse=True)
def _bounds_and_guards(request):
    """Under the bounds-checked build (GLM53_BOUNDS=1) every GPU test ends with no out-of-range index recorded by
    a kernel and every guard band around the runtimes' scratch buffers intact."""
    if os.environ.get("GLM53_BOUNDS", "0") != "1" or not request.node.get_closest_marker("gpu"):
        yield
        return
    import torch
    from glm53.ops import _ext
    from glm53.utils import canary
    mod = _ext.require()
    torch.cuda.synchronize()
    mod.bounds_reset()
    yield
    torch.cuda.synchronize()
    enabled, fails = mod.bounds_status()
    bad = canary.check_all()
    mod.bounds_reset()
    assert enabled, "GLM53_BOUNDS=1 but the loaded extension was built without bounds checks"
    assert not fails, f"out-of-range device indices (code, index, limit, count): {fails}"
    assert not bad, f"guard bands overwritten: {bad}"


@pytest.fixture(scope="session")
def tiny_cfg():
    import glm53
    return glm53.tiny_config()


@pytest.fixture(scope="session")
def tiny_ckpt(tiny_cfg):
    from glm53.models import weights as W
    return W.random_checkpoint(tiny_cfg, seed=0)


@pytest.fixture(scope="session")
def tiny_weights(tiny_cfg, tiny_ckpt):
    from glm53.models import weights as W
    return W.prepare(W.DictSource(tiny_ckpt), tiny_cfg)
