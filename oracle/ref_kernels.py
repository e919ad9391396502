"""The reference's own CUDA kernels as the exact GPU oracle -- TEST INFRASTRUCTURE ONLY.

``oracle/Makefile`` (target ``ref``) compiles the reference's src/kernels.cu, unchanged and
read where it lies, for sm_100a together with ``oracle/ref_abi.cu`` into
``oracle/_ref/libqwen3_ref.so``. This module binds it with ctypes. Pointer arguments are
device addresses (ints); ``stream`` is a ``cudaStream_t`` as an int (0 = legacy stream).

Only the GPU parity tests and the golden-fixture generator use it, as the checker.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_LIB = HERE / "_ref" / "libqwen3_ref.so"
REF_ENGINE = HERE / "_ref" / "ref_engine"

_lib = None


def available() -> bool:
    return REF_LIB.exists()


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(str(REF_LIB))
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sigs = {
            "ref_embedding_forward": [P, P, P, I, P],
            "ref_rmsnorm_forward": [P, P, P, I, I, F, P],
            "ref_gemv_forward": [P, P, P, I, I, P],
            "ref_gemv_residual_forward": [P, P, P, I, I, P, P],
            "ref_qkv_forward": [P, P, P, P, P, P, P, I, I, I, P],
            "ref_gate_up_forward": [P, P, P, P, I, I, P, P, P],
            "ref_qk_norm_rope_forward": [P, P, P, P, P, P, P, P, I, I, I, F, F, P, P, P],
            "ref_attention_forward": [P, P, P, P, P, I, I, I, P, I, F, P],
            "ref_argmax_forward": [P, P, I, P],
            "ref_sample_forward": [P, P, I, F, F, P],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = I
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    err = getattr(lib(), "ref_" + name)(*args)
    if err != 0:
        raise RuntimeError(f"reference kernel {name} failed with CUDA error {err}")
