"""The C ABI library, without a GPU: it loads, and exports every entry point the header
declares plus the reference's C++ launcher names (the drop-in symbols)."""
import ctypes
import subprocess
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import conftest  # noqa: E402,F401
from llm_inference_b200 import _lib, build  # noqa: E402

# src/kernels.cuh:7-26, demangled
REFERENCE_LAUNCHERS = [
    "embedding_forward(__nv_bfloat16*, __nv_bfloat16 const*, int const*, int, CUstream_st*)",
    "rmsnorm_forward(__nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, int, int, float, CUstream_st*)",
    "gemv_forward(__nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, int, int, CUstream_st*)",
    "gemv_residual_forward(__nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, int, int, "
    "__nv_bfloat16*, CUstream_st*)",
    "qkv_forward(__nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, "
    "__nv_bfloat16 const*, __nv_bfloat16 const*, int, int, int, CUstream_st*)",
    "gate_up_forward(__nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, __nv_bfloat16 const*, int, int, "
    "__nv_bfloat16*, __nv_bfloat16*, CUstream_st*)",
    "qk_norm_rope_forward(__nv_bfloat16*, __nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, "
    "__nv_bfloat16 const*, __nv_bfloat16*, __nv_bfloat16*, int const*, int, int, int, float, float, "
    "__nv_bfloat16*, __nv_bfloat16*, CUstream_st*)",
    "attention_forward(__nv_bfloat16*, __nv_bfloat16 const*, __nv_bfloat16 const*, __nv_bfloat16 const*, float*, "
    "int, int, int, int const*, int, float, CUstream_st*)",
    "argmax_forward(int*, __nv_bfloat16 const*, int, CUstream_st*)",
    "sample_forward(int*, __nv_bfloat16 const*, int, float, float, CUstream_st*)",
]


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    names = [line.split()[-1] for line in out.splitlines() if " T " in line]
    dem = subprocess.run(["c++filt"], input="\n".join(names), capture_output=True, text=True,
                         check=True).stdout.splitlines()
    return set(names), set(dem)


def test_header_entry_points_are_exported(lib):
    declared = _lib.header_functions()
    assert len(declared) >= 13
    raw, _ = _exported()
    missing = [f for f in declared if f not in raw]
    assert not missing, missing
    for f in declared:
        assert hasattr(lib, f)
    assert set(declared) == set(_lib.SIGNATURES), "SIGNATURES and the header disagree"


def test_reference_launcher_names_are_exported(lib):
    _, demangled = _exported()
    missing = [f for f in REFERENCE_LAUNCHERS if f not in demangled]
    assert not missing, missing


def test_status_strings(lib):
    assert lib.q3_status_string(0) == b"ok"
    for code in range(1, 6):
        assert lib.q3_status_string(code) not in (b"ok", b"unknown status")
    assert lib.q3_status_string(99) == b"unknown status"
