"""ctypes binding of libqwen3_b200.so (include/qwen3_b200.h).

The library must exist (built by build.py, in-tree under _build/); there is no fallback.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

from . import build as _build

LIB_PATH = _build.LIB
HEADER = _build.INCLUDE / "qwen3_b200.h"


class Q3Error(RuntimeError):
    """A q3_* entry point returned a status other than Q3_OK."""

    def __init__(self, name: str, status: int, detail: str = ""):
        self.status = status
        super().__init__(f"{name}: {detail}" if detail else f"{name}: status {status}")


_P, _I, _F, _LL, _U = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_uint

# argument types of every entry point, in header order
SIGNATURES: dict[str, list] = {
    "q3_status_string": [_I],
    "q3_last_cuda_error": [],
    "q3_device_error": [_P, ctypes.POINTER(_U)],
    "q3_selftest_wait_timeout": [_P, _P],
    "q3_embedding_forward": [_P, _P, _P, _I, _P],
    "q3_rmsnorm_forward": [_P, _P, _P, _I, _I, _F, _P],
    "q3_gemv_forward": [_P, _P, _P, _I, _I, _P],
    "q3_gemv_residual_forward": [_P, _P, _P, _I, _I, _P, _P],
    "q3_qkv_forward": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P],
    "q3_gate_up_forward": [_P, _P, _P, _P, _I, _I, _P, _P, _P],
    "q3_qk_norm_rope_forward": [_P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _F, _F, _P, _P, _P],
    "q3_attention_forward": [_P, _P, _P, _P, _P, _I, _I, _I, _P, _I, _F, _P],
    "q3_argmax_forward": [_P, _P, _I, _P],
    "q3_sample_forward": [_P, _P, _I, _F, _F, _P],
    "q3_embedding_batched": [_P, _P, _P, _I, _I, _I, _P],
    "q3_gemv_batched": [_P, _P, _P, _I, _I, _I, _P],
    "q3_gemv_residual_batched": [_P, _P, _P, _I, _I, _I, _P, _P],
    "q3_qkv_batched": [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P],
    "q3_gate_up_batched": [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P],
    "q3_qk_norm_rope_batched": [_P, _P, _P, _P, _P, _P, _P, _LL, _LL, _LL, _P, _I, _I, _I, _I, _I, _F, _F, _P, _P, _P],
    "q3_attention_scratch_bytes": [_I, _I, _I, _I, _I],
    "q3_attention_batched": [_P, _P, _P, _P, _LL, _LL, _LL, _P, _P, _I, _I, _I, _I, _I, _F, _P],
    "q3_attention_batched_static": [_P, _P, _P, _P, _LL, _LL, _LL, _P, _I, _I, _I, _I, _I, _F, _P],
    "q3_rope_attention_chunks": [_I, _I, _I, _I, _I],
    "q3_rope_attention_batched": [_P, _P, _P, _P, _P, _P, _P, _P, _LL, _LL, _LL, _P, _I, _I, _I, _I, _I, _F, _F, _F,
                                  _I, _P],
    "q3_argmax_batched": [_P, _P, _I, _I, _P],
    "q3_fill_normal_bf16": [_P, _LL, ctypes.c_ulonglong, _F, _F, _P],
    "q3_weight_bytes_per_step": [_P],
    "q3_kv_bytes_per_position": [_P],
    "q3_engine_create": [_P, _P, _I, _I, _I, _I, _P, _P],
    "q3_engine_destroy": [_P],
    "q3_engine_capture": [_P],
    "q3_engine_step": [_P, _I],
    "q3_engine_set_state": [_P, _P, _P],
    "q3_engine_forward": [_P, _P, _P],
    "q3_engine_sample_argmax": [_P, _P],
    "q3_engine_prefill": [_P, _I, _P, _I, _I],
    "q3_engine_fill_kv_normal": [_P, _I, ctypes.c_ulonglong],
    "q3_engine_info": [_P, _P],
}
RESTYPES = {"q3_status_string": ctypes.c_char_p, "q3_attention_scratch_bytes": ctypes.c_size_t,
            "q3_weight_bytes_per_step": ctypes.c_size_t, "q3_kv_bytes_per_position": ctypes.c_size_t}

_lib = None


def header_functions() -> list[str]:
    """Names of the functions include/qwen3_b200.h declares."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return re.findall(r"\b(q3_\w+)\s*\(", text)


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(f"{LIB_PATH} is missing: run `python llm-inference_b200/build.py` "
                                    "(or __graft_entry__.build()) first")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, _I)
        _lib = lib
    return _lib


def check(name: str, status: int) -> None:
    if status != 0:
        lib = load()
        detail = lib.q3_status_string(status).decode()
        if status == 3:
            detail += f" (cudaError {lib.q3_last_cuda_error()})"
        raise Q3Error(name, status, detail)


def call(name: str, *args) -> None:
    check(name, getattr(load(), name)(*args))
