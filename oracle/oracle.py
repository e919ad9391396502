"""CPU oracle for the Qwen3 decode kernels -- TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline leg may import this
module, and only as the checker. It wraps ``qwen3_oracle.c`` (a plain-C restatement of the
reference's src/kernels.cu, built into ``oracle/_build/liboracle.so`` by ``oracle/Makefile``)
and strings those kernels together in the launch order of the reference's
``forward_kernels`` (src/forward.cu:118-193), producing the same named intermediate tensors
as the reference's dump path (src/forward.cu:125-192, ref/dump.py:39-63).

bf16 tensors are numpy ``uint16`` arrays holding the raw bits.
"""
from __future__ import annotations

import ctypes
import json
import math
import os
import struct
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib = None


def build() -> Path:
    """Compile the C restatement (gcc, a second or so)."""
    subprocess.run(["make", "-s", "all"], cwd=HERE, check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sigs = {
            "oracle_embedding": [P, P, I, I],
            "oracle_rmsnorm": [P, P, P, I, I, F],
            "oracle_gemv": [P, P, P, I, I],
            "oracle_gemv_residual": [P, P, P, I, I, P],
            "oracle_qkv": [P, P, P, P, P, P, P, I, I, I],
            "oracle_gate_up": [P, P, P, P, I, I, P, P],
            "oracle_qk_norm_rope": [P, P, P, P, P, P, P, I, I, I, I, F, F, P, P],
            "oracle_attention": [P, P, P, P, I, I, I, I, F],
            "oracle_scores": [P, P, P, I, I, I, I, F],
            "oracle_argmax": [P, I],
            "oracle_sample": [P, I, F, F],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = I if name in ("oracle_argmax", "oracle_sample") else None
        _lib = L
    return _lib


# ---------------------------------------------------------------- bf16 helpers

def f32_to_bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits, NaN -> 0x7fff (as cvt.rn.bf16.f32)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[(u & 0x7FFFFFFF) > 0x7F800000] = 0x7FFF
    return r


def bf16_to_f32(b) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def ulp_diff(a, b) -> np.ndarray:
    """Distance in bf16 units in the last place between two arrays of bf16 bits."""
    def key(x):
        x = np.asarray(x, dtype=np.uint16).astype(np.int32)
        mag = x & 0x7FFF
        return np.where(x & 0x8000, -mag, mag)
    return np.abs(key(a) - key(b))


def randn_bf16(rng: np.random.Generator, shape, std=1.0, mean=0.0) -> np.ndarray:
    return f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(std) + np.float32(mean))


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- kernel restatements

def embedding(table, token, hidden):
    out = np.empty(hidden, np.uint16)
    lib().oracle_embedding(_p(out), _p(table), int(token), int(hidden))
    return out


def rmsnorm(x, weight, eps):
    x = np.ascontiguousarray(x, np.uint16)
    dim = x.shape[-1]
    rows = x.size // dim
    out = np.empty_like(x)
    lib().oracle_rmsnorm(_p(out), _p(x), _p(weight), rows, dim, float(eps))
    return out


def gemv(w, x):
    rows, cols = w.shape
    out = np.empty(rows, np.uint16)
    lib().oracle_gemv(_p(out), _p(w), _p(x), rows, cols)
    return out


def gemv_residual(x, w, inp, want_tap=False):
    """Returns (new x, tap). ``x`` is not modified."""
    rows, cols = w.shape
    x = np.array(x, np.uint16, copy=True)
    tap = np.empty(rows, np.uint16) if want_tap else None
    lib().oracle_gemv_residual(_p(x), _p(w), _p(inp), rows, cols, _p(tap))
    return x, tap


def qkv(wq, wk, wv, x):
    q_rows, cols = wq.shape
    kv_rows = wk.shape[0]
    q = np.empty(q_rows, np.uint16)
    k = np.empty(kv_rows, np.uint16)
    v = np.empty(kv_rows, np.uint16)
    lib().oracle_qkv(_p(q), _p(k), _p(v), _p(wq), _p(wk), _p(wv), _p(x), q_rows, kv_rows, cols)
    return q, k, v


def gate_up(w_gate, w_up, x, want_taps=False):
    rows, cols = w_gate.shape
    act = np.empty(rows, np.uint16)
    gt = np.empty(rows, np.uint16) if want_taps else None
    ut = np.empty(rows, np.uint16) if want_taps else None
    lib().oracle_gate_up(_p(act), _p(w_gate), _p(w_up), _p(x), rows, cols, _p(gt), _p(ut))
    return act, gt, ut


def qk_norm_rope(q, k, v, q_norm_w, k_norm_w, key_cache, value_cache, pos, n_heads, n_kv_heads,
                 head_dim, eps, theta, want_taps=False):
    """In place on q, k (copies returned) and on the caches (modified in place)."""
    q = np.array(q, np.uint16, copy=True)
    k = np.array(k, np.uint16, copy=True)
    qt = np.empty_like(q) if want_taps else None
    kt = np.empty_like(k) if want_taps else None
    lib().oracle_qk_norm_rope(_p(q), _p(k), _p(np.ascontiguousarray(v)), _p(q_norm_w), _p(k_norm_w),
                              _p(key_cache), _p(value_cache), int(pos), n_heads, n_kv_heads,
                              head_dim, float(eps), float(theta), _p(qt), _p(kt))
    return q, k, qt, kt


def attention(q, key_cache, value_cache, n_heads, n_kv_heads, head_dim, pos, scale=None):
    if scale is None:
        scale = float(np.float32(1.0 / math.sqrt(head_dim)))
    out = np.empty(n_heads * head_dim, np.uint16)
    lib().oracle_attention(_p(out), _p(np.ascontiguousarray(q)), _p(key_cache), _p(value_cache),
                           n_heads, n_kv_heads, head_dim, int(pos), float(scale))
    return out


def scores(q, key_cache, n_heads, n_kv_heads, head_dim, pos, scale):
    """[n_heads][pos + 1] float32 attention scores, the reference's rounding (src/kernels.cu:450-461)."""
    out = np.empty((n_heads, pos + 1), np.float32)
    lib().oracle_scores(_p(out), _p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(key_cache)), n_heads,
                        n_kv_heads, head_dim, int(pos), float(scale))
    return out


def argmax(x):
    x = np.ascontiguousarray(x, np.uint16)
    return int(lib().oracle_argmax(_p(x), x.size))


def sample(x, inv_temp, u):
    x = np.ascontiguousarray(x, np.uint16)
    return int(lib().oracle_sample(_p(x), x.size, float(inv_temp), float(u)))


# ---------------------------------------------------------------- checkpoint reading

def read_safetensors(path) -> dict[str, np.ndarray]:
    """Minimal reader: ``[u64 header length][JSON header][data]`` (src/loader.cu:141-180)."""
    raw = Path(path).read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        assert meta["dtype"] == "BF16", name
        b, e = meta["data_offsets"]
        out[name] = np.frombuffer(data[b:e], dtype=np.uint16).reshape(meta["shape"]).copy()
    return out


def load_model(model_dir) -> tuple[dict, dict]:
    model_dir = Path(model_dir)
    cfg = json.loads((model_dir / "config.json").read_text())
    tensors = {}
    for p in sorted(model_dir.glob("*.safetensors")):
        tensors.update(read_safetensors(p))
    return cfg, tensors


# ---------------------------------------------------------------- forward pass

class OracleModel:
    """Batch-1 decode over a small model in the reference's launch order.

    ``forward(token, pos)`` follows src/forward.cu:118-193 (``forward_kernels``) with a
    contiguous per-layer cache of ``max_seq`` positions (src/forward.cuh:15-16) and
    returns the logits; ``taps`` then holds every dumped tensor of that position under the
    reference's names (src/forward.cu:125-192).
    """

    def __init__(self, cfg: dict, tensors: dict, max_seq: int | None = None):
        self.cfg = cfg
        self.t = tensors
        self.hidden = cfg["hidden_size"]
        self.inter = cfg["intermediate_size"]
        self.n_layers = cfg["num_hidden_layers"]
        self.n_heads = cfg["num_attention_heads"]
        self.n_kv = cfg["num_key_value_heads"]
        self.head_dim = cfg["head_dim"]
        self.vocab = cfg["vocab_size"]
        self.eps = float(np.float32(cfg["rms_norm_eps"]))
        self.theta = float(np.float32(cfg["rope_theta"]))
        self.max_seq = max_seq or min(cfg["max_position_embeddings"], 4096)
        kv_dim = self.n_kv * self.head_dim
        self.kcache = np.zeros((self.n_layers, self.max_seq, kv_dim), np.uint16)
        self.vcache = np.zeros((self.n_layers, self.max_seq, kv_dim), np.uint16)
        self.scale = float(np.float32(1.0 / math.sqrt(self.head_dim)))
        self.lm_head = tensors.get("lm_head.weight") if not cfg["tie_word_embeddings"] else None
        if self.lm_head is None:
            self.lm_head = tensors["model.embed_tokens.weight"]
        self.taps: dict[str, np.ndarray] = {}

    def _w(self, l, suffix):
        return self.t[f"model.layers.{l}.{suffix}"]

    def forward(self, token: int, pos: int) -> np.ndarray:
        taps = {}
        x = embedding(self.t["model.embed_tokens.weight"], token, self.hidden)
        taps["embed"] = x.copy()
        for l in range(self.n_layers):
            p = f"L{l:02d}"
            xb = rmsnorm(x, self._w(l, "input_layernorm.weight"), self.eps)
            taps[f"{p}.attn_norm"] = xb
            q, k, v = qkv(self._w(l, "self_attn.q_proj.weight"), self._w(l, "self_attn.k_proj.weight"),
                          self._w(l, "self_attn.v_proj.weight"), xb)
            taps[f"{p}.q_proj"], taps[f"{p}.k_proj"], taps[f"{p}.v_proj"] = q, k, v
            q, k, qt, kt = qk_norm_rope(q, k, v, self._w(l, "self_attn.q_norm.weight"),
                                        self._w(l, "self_attn.k_norm.weight"), self.kcache[l],
                                        self.vcache[l], pos, self.n_heads, self.n_kv,
                                        self.head_dim, self.eps, self.theta, want_taps=True)
            taps[f"{p}.q_norm"], taps[f"{p}.k_norm"] = qt, kt
            taps[f"{p}.q_rope"], taps[f"{p}.k_rope"] = q, k
            att = attention(q, self.kcache[l], self.vcache[l], self.n_heads, self.n_kv,
                            self.head_dim, pos, self.scale)
            taps[f"{p}.attn_out"] = att
            x, o = gemv_residual(x, self._w(l, "self_attn.o_proj.weight"), att, want_tap=True)
            taps[f"{p}.o_proj"], taps[f"{p}.attn_resid"] = o, x.copy()
            xb = rmsnorm(x, self._w(l, "post_attention_layernorm.weight"), self.eps)
            taps[f"{p}.mlp_norm"] = xb
            hb, g, u = gate_up(self._w(l, "mlp.gate_proj.weight"), self._w(l, "mlp.up_proj.weight"),
                               xb, want_taps=True)
            taps[f"{p}.gate"], taps[f"{p}.up"], taps[f"{p}.mlp_act"] = g, u, hb
            x, d = gemv_residual(x, self._w(l, "mlp.down_proj.weight"), hb, want_tap=True)
            taps[f"{p}.down"], taps[f"{p}.out"] = d, x.copy()
        xb = rmsnorm(x, self.t["model.norm.weight"], self.eps)
        taps["final_norm"] = xb
        logits = gemv(self.lm_head, xb)
        taps["logits"] = logits
        self.taps = taps
        return logits

    def greedy(self, prompt: list[int], n_new: int) -> tuple[list[int], list[np.ndarray]]:
        """Prompt one position at a time (src/main.cu:328-330), then greedy tokens."""
        logits = None
        all_logits = []
        for pos, tok in enumerate(prompt):
            logits = self.forward(tok, pos)
            all_logits.append(logits)
        out = []
        pos = len(prompt)
        for i in range(n_new):
            tok = argmax(logits)
            out.append(tok)
            if i + 1 < n_new:
                logits = self.forward(tok, pos)
                all_logits.append(logits)
                pos += 1
        return out, all_logits
