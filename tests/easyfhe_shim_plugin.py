"""pytest plugin: run the reference's own test files on this engine.

``python -m pytest -p tests.easyfhe_shim_plugin baseline/_ref/tests/<file>`` puts the reference install
(``baseline/_ref``: its ``llama3fhe`` package and, copied beside it, its ``tests/``) on the path and registers
``holmes_b200`` under the import name ``easyfhe`` (:func:`holmes_b200.easyfhe_compat.install`) before the reference's
conftest or test modules import anything, so the reference's operators and tests run unchanged over libholmes_cuda.
"""
from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")


def pytest_configure(config):
    for path in (REF, ROOT):
        if path not in sys.path:
            sys.path.insert(0, path)
    from holmes_b200 import easyfhe_compat

    easyfhe_compat.install()
