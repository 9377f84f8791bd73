"""Import shim: ``import glm53`` loads the package that lives in
``glm-5.3-flash-dgx-spark-vllm-optimization_b200/`` (a directory name that is not a valid Python identifier).

The module replaces itself in ``sys.modules`` with that package, so ``import glm53.models.reference`` and the
package's relative imports resolve inside the directory.
"""

from __future__ import annotations

import importlib.util
import os
import sys

_PKG_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "glm-5.3-flash-dgx-spark-vllm-optimization_b200")


def _load():
    spec = importlib.util.spec_from_file_location(__name__, os.path.join(_PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[_PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[__name__] = mod
    spec.loader.exec_module(mod)
    return mod


_load()
