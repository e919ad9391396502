"""llm_inference_b200: sm_100a (B200) decode kernels for Qwen3.

A drop-in for the kernels of William-Lamer/llm-inference (src/kernels.cuh), exported by
libqwen3_b200.so through the C ABI in include/qwen3_b200.h, plus a batched, data-parallel
decode host.

The functions below mirror the reference launchers one for one (same names and argument
order) for callers holding torch CUDA tensors; bf16 tensors are torch.bfloat16, position and
token buffers torch.int32, and ``stream`` defaults to torch's current stream. Errors raise
:class:`Q3Error` where the reference would print and exit.
"""
from __future__ import annotations

from ._lib import Q3Error, call, load  # noqa: F401

__all__ = [
    "Q3Error", "load", "embedding_forward", "rmsnorm_forward", "gemv_forward",
    "gemv_residual_forward", "qkv_forward", "gate_up_forward", "qk_norm_rope_forward",
    "attention_forward", "argmax_forward", "sample_forward", "device_error",
]


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(stream):
    if stream is not None:
        return stream
    import torch
    return torch.cuda.current_stream().cuda_stream


def embedding_forward(out, table, d_token, hidden, stream=None):
    call("q3_embedding_forward", _ptr(out), _ptr(table), _ptr(d_token), hidden, _stream(stream))


def rmsnorm_forward(out, inp, weight, rows, dim, eps, stream=None):
    call("q3_rmsnorm_forward", _ptr(out), _ptr(inp), _ptr(weight), rows, dim, eps, _stream(stream))


def gemv_forward(out, w, x, rows, cols, stream=None):
    call("q3_gemv_forward", _ptr(out), _ptr(w), _ptr(x), rows, cols, _stream(stream))


def gemv_residual_forward(x, w, inp, rows, cols, tap=None, stream=None):
    call("q3_gemv_residual_forward", _ptr(x), _ptr(w), _ptr(inp), rows, cols, _ptr(tap), _stream(stream))


def qkv_forward(q, k, v, wq, wk, wv, x, q_rows, kv_rows, cols, stream=None):
    call("q3_qkv_forward", _ptr(q), _ptr(k), _ptr(v), _ptr(wq), _ptr(wk), _ptr(wv), _ptr(x),
         q_rows, kv_rows, cols, _stream(stream))


def gate_up_forward(act, w_gate, w_up, x, rows, cols, gate_tap=None, up_tap=None, stream=None):
    call("q3_gate_up_forward", _ptr(act), _ptr(w_gate), _ptr(w_up), _ptr(x), rows, cols,
         _ptr(gate_tap), _ptr(up_tap), _stream(stream))


def qk_norm_rope_forward(q, k, v, q_norm_w, k_norm_w, key_cache, value_cache, d_pos, n_heads,
                         n_kv_heads, head_dim, eps, theta, q_tap=None, k_tap=None, stream=None):
    call("q3_qk_norm_rope_forward", _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm_w), _ptr(k_norm_w),
         _ptr(key_cache), _ptr(value_cache), _ptr(d_pos), n_heads, n_kv_heads, head_dim, eps, theta,
         _ptr(q_tap), _ptr(k_tap), _stream(stream))


def attention_forward(out, q, key_cache, value_cache, att, n_heads, n_kv_heads, head_dim, d_pos,
                      max_seq, scale, stream=None):
    call("q3_attention_forward", _ptr(out), _ptr(q), _ptr(key_cache), _ptr(value_cache), _ptr(att),
         n_heads, n_kv_heads, head_dim, _ptr(d_pos), max_seq, scale, _stream(stream))


def argmax_forward(out, x, n, stream=None):
    call("q3_argmax_forward", _ptr(out), _ptr(x), n, _stream(stream))


def sample_forward(out, x, n, inv_temp, u, stream=None):
    call("q3_sample_forward", _ptr(out), _ptr(x), n, inv_temp, u, _stream(stream))


def device_error(stream=None) -> int:
    """Read and clear the kernels' device error flags (synchronizes the stream)."""
    import ctypes
    flags = ctypes.c_uint(0)
    call("q3_device_error", _stream(stream), ctypes.byref(flags))
    return flags.value
