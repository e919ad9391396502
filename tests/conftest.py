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


def pytest_terminal_summary(terminalreporter):
    """The parity statistics the GPU tests recorded (tests/parity.py): per compared tensor, the
    maximum bf16 ulp distance from the reference and how many elements are more than 1 ulp away."""
    import json
    import os

    parity = sys.modules.get("parity")
    tr = terminalreporter
    for m in getattr(parity, "MEASURES", []):
        tr.write_line(f"measured: {m}")
    recs = getattr(parity, "RECORDS", None)
    if not recs:
        return
    tr.write_sep("-", f"parity: {len(recs)} comparisons (max ulp, elements > 1 ulp, not identical)")
    worst = sorted(recs, key=lambda r: (-r["max_ulp"], -r["over_1ulp"]))
    for r in worst[:40]:
        tr.write_line(f"{r['max_ulp']:6d} {r['over_1ulp']:9d} {r['not_identical']:9d} / {r['elements']:<10d} "
                      f"{r['what']}  [{r['bar']}]")
    path = os.environ.get("Q3_PARITY_LOG")
    if path:
        with open(path, "w") as f:
            for r in recs:
                f.write(json.dumps(r) + "\n")
