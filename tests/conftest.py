"""Shared test set-up: the ``gpu`` marker, the package loader and common fixtures."""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "llm-inference_b200"
for _p in (ROOT, ROOT / "oracle", ROOT / "tests" / "golden"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))


def load_package():
    """Import the package directory ``llm-inference_b200`` as ``llm_inference_b200``."""
    name = "llm_inference_b200"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(
            name, PKG_DIR / "__init__.py", submodule_search_locations=[str(PKG_DIR)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
