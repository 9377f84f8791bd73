import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


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
