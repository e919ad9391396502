"""Kernel parity cases shared by the golden-fixture generator and the tests.

Each case is (kind, name, params). ``inputs(kind, params)`` rebuilds its inputs
deterministically from ``params["seed"]`` (numpy PCG64), so fixtures store only outputs. The
value distributions follow the benchmark configurations: weights N(0, 0.02), norm weights
1 + N(0, 0.02), activations, caches and logits N(0, 1); token ids and positions as given.
Shapes cover the Qwen3-1.7B/4B sizes of the microbenchmark configuration plus edge cases:
ragged column counts, row counts that leave CTAs uneven, position 0 and the last cache row,
head_dim 64 and 256, GQA group sizes 1, 2 and 4, argmax ties, NaNs and all -inf rows, and
sampling coins at 0 and near 1.

``run(impl, kind, params, inp)`` executes one case with impl in
  "oracle": the C restatement (CPU),
  "ref":    the reference's own kernels compiled for sm_100a (oracle/_ref, GPU),
  "mine":   libqwen3_b200.so through its C ABI (GPU),
and returns a dict of numpy outputs (bf16 as uint16 bits, ints as int32).
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as O  # noqa: E402

W_STD = 0.02


def _c(kind, name, seed, **p):
    p["seed"] = seed
    return (kind, name, p)


CASES = [
    _c("embedding", "emb_2048", 1, vocab=1000, hidden=2048, token=777),
    _c("embedding", "emb_ragged_hidden", 2, vocab=50, hidden=100, token=49),
    _c("rmsnorm", "rms_4x2048", 3, rows=4, dim=2048),
    _c("rmsnorm", "rms_1x2560", 4, rows=1, dim=2560),
    _c("rmsnorm", "rms_3x1000", 5, rows=3, dim=1000),
    _c("gemv", "gemv_1000x2048", 6, rows=1000, cols=2048),
    _c("gemv", "gemv_77x136", 7, rows=77, cols=136),
    _c("gemv", "gemv_5x8", 8, rows=5, cols=8),
    _c("gemv", "gemv_3000x2600", 9, rows=3000, cols=2600),
    _c("gemv_residual", "res_2048x6144", 10, rows=2048, cols=6144),
    _c("gemv_residual", "res_64x72", 11, rows=64, cols=72),
    _c("gemv_residual", "res_300x2600", 12, rows=300, cols=2600),
    _c("qkv", "qkv_2048_1024_2048", 13, q_rows=2048, kv_rows=1024, cols=2048),
    _c("qkv", "qkv_256_128_256", 14, q_rows=256, kv_rows=128, cols=256),
    _c("gate_up", "gu_6144x2048", 15, rows=6144, cols=2048),
    _c("gate_up", "gu_100x264", 16, rows=100, cols=264),
    _c("gate_up", "gu_9728x2560", 17, rows=9728, cols=2560),
    _c("qk_norm_rope", "rope_pos0", 18, n_heads=16, n_kv=8, hd=128, pos=0, max_seq=8),
    _c("qk_norm_rope", "rope_pos1000", 19, n_heads=16, n_kv=8, hd=128, pos=1000, max_seq=1024),
    _c("qk_norm_rope", "rope_pos4095", 20, n_heads=32, n_kv=8, hd=128, pos=4095, max_seq=4096),
    _c("qk_norm_rope", "rope_hd64", 21, n_heads=4, n_kv=2, hd=64, pos=37, max_seq=64),
    _c("qk_norm_rope", "rope_hd256_far", 22, n_heads=2, n_kv=1, hd=256, pos=100000, max_seq=100001),
    _c("attention", "att_pos0", 23, n_heads=16, n_kv=8, hd=128, pos=0, max_seq=512),
    _c("attention", "att_pos300", 24, n_heads=16, n_kv=8, hd=128, pos=300, max_seq=512),
    _c("attention", "att_pos511", 25, n_heads=16, n_kv=8, hd=128, pos=511, max_seq=512),
    _c("attention", "att_gqa4_pos1000", 26, n_heads=32, n_kv=8, hd=128, pos=1000, max_seq=1024),
    _c("attention", "att_hd64", 27, n_heads=4, n_kv=2, hd=64, pos=100, max_seq=128),
    _c("attention", "att_mha_hd256", 28, n_heads=2, n_kv=2, hd=256, pos=70, max_seq=80),
    _c("attention", "att_pos4095", 29, n_heads=16, n_kv=8, hd=128, pos=4095, max_seq=4096),
    _c("argmax", "argmax_tie", 30, n=151936, plant="tie"),
    _c("argmax", "argmax_nan", 31, n=151936, plant="nan"),
    _c("argmax", "argmax_all_neg_inf", 32, n=1000, plant="neg_inf"),
    _c("argmax", "argmax_n7", 33, n=7, plant="none"),
    _c("argmax", "argmax_odd_tail", 34, n=151937, plant="last"),
    _c("sample", "sample_t1", 35, n=151936, inv_temp=1.0, u=0.3),
    _c("sample", "sample_t07", 36, n=151936, inv_temp=1.0 / 0.7, u=0.999),
    _c("sample", "sample_u0", 37, n=151936, inv_temp=1.0, u=0.0),
]


def case(name):
    for c in CASES:
        if c[1] == name:
            return c
    raise KeyError(name)


def inputs(kind: str, p: dict) -> dict:
    rng = np.random.default_rng(p["seed"])
    rn = lambda *shape, std=1.0, mean=0.0: O.randn_bf16(rng, shape, std, mean)  # noqa: E731
    if kind == "embedding":
        return {"table": rn(p["vocab"], p["hidden"]), "token": np.array([p["token"]], np.int32)}
    if kind == "rmsnorm":
        return {"x": rn(p["rows"], p["dim"]), "w": rn(p["dim"], std=W_STD, mean=1.0)}
    if kind in ("gemv",):
        return {"w": rn(p["rows"], p["cols"], std=W_STD), "x": rn(p["cols"])}
    if kind == "gemv_residual":
        return {"w": rn(p["rows"], p["cols"], std=W_STD), "inp": rn(p["cols"]), "x": rn(p["rows"])}
    if kind == "qkv":
        return {"wq": rn(p["q_rows"], p["cols"], std=W_STD), "wk": rn(p["kv_rows"], p["cols"], std=W_STD),
                "wv": rn(p["kv_rows"], p["cols"], std=W_STD), "x": rn(p["cols"])}
    if kind == "gate_up":
        return {"wg": rn(p["rows"], p["cols"], std=W_STD), "wu": rn(p["rows"], p["cols"], std=W_STD),
                "x": rn(p["cols"])}
    if kind == "qk_norm_rope":
        hd = p["hd"]
        return {"q": rn(p["n_heads"] * hd), "k": rn(p["n_kv"] * hd), "v": rn(p["n_kv"] * hd),
                "qn": rn(hd, std=W_STD, mean=1.0), "kn": rn(hd, std=W_STD, mean=1.0),
                "pos": np.array([p["pos"]], np.int32)}
    if kind == "attention":
        hd, kvd = p["hd"], p["n_kv"] * p["hd"]
        return {"q": rn(p["n_heads"] * hd), "kc": rn(p["max_seq"], kvd), "vc": rn(p["max_seq"], kvd),
                "pos": np.array([p["pos"]], np.int32)}
    if kind == "argmax":
        x = rng.standard_normal(p["n"], dtype=np.float32)
        n = p["n"]
        if p["plant"] == "tie":
            x[[5000, 100000, 151935]] = 9.0
        elif p["plant"] == "nan":
            x[[0, 77, 140000]] = np.nan
            x[120000] = 8.0
        elif p["plant"] == "neg_inf":
            x[:] = -np.inf
        elif p["plant"] == "last":
            x[n - 1] = 20.0
        return {"x": O.f32_to_bf16(x)}
    if kind == "sample":
        return {"x": O.randn_bf16(rng, (p["n"],), 3.0)}
    raise ValueError(kind)


# ------------------------------------------------------------------ CPU oracle

def run_oracle(kind: str, p: dict, inp: dict) -> dict:
    if kind == "embedding":
        return {"out": O.embedding(inp["table"], int(inp["token"][0]), p["hidden"])}
    if kind == "rmsnorm":
        return {"out": O.rmsnorm(inp["x"], inp["w"], 1e-6)}
    if kind == "gemv":
        return {"out": O.gemv(inp["w"], inp["x"])}
    if kind == "gemv_residual":
        x, tap = O.gemv_residual(inp["x"], inp["w"], inp["inp"], want_tap=True)
        return {"x": x, "tap": tap}
    if kind == "qkv":
        q, k, v = O.qkv(inp["wq"], inp["wk"], inp["wv"], inp["x"])
        return {"q": q, "k": k, "v": v}
    if kind == "gate_up":
        act, g, u = O.gate_up(inp["wg"], inp["wu"], inp["x"], want_taps=True)
        return {"act": act, "gate": g, "up": u}
    if kind == "qk_norm_rope":
        kvd = p["n_kv"] * p["hd"]
        # the kernel touches only row `pos`: a one-row cache view at that row stands in
        kc = np.zeros((p["pos"] + 1, kvd), np.uint16)
        vc = np.zeros((p["pos"] + 1, kvd), np.uint16)
        q, k, qt, kt = O.qk_norm_rope(inp["q"], inp["k"], inp["v"], inp["qn"], inp["kn"], kc, vc, p["pos"],
                                      p["n_heads"], p["n_kv"], p["hd"], 1e-6, 1e6, want_taps=True)
        return {"q": q, "k": k, "q_tap": qt, "k_tap": kt, "krow": kc[p["pos"]], "vrow": vc[p["pos"]]}
    if kind == "attention":
        return {"out": O.attention(inp["q"], inp["kc"], inp["vc"], p["n_heads"], p["n_kv"], p["hd"], p["pos"])}
    if kind == "argmax":
        return {"out": np.array([O.argmax(inp["x"])], np.int32)}
    if kind == "sample":
        return {"out": np.array([O.sample(inp["x"], p["inv_temp"], p["u"])], np.int32)}
    raise ValueError(kind)


# ------------------------------------------------------------------ GPU runners

def _dev(a):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(a.copy()).cuda()


def _host(t):
    import torch
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def _launcher(impl: str):
    if impl == "ref":
        import ref_kernels
        return lambda name, *args: ref_kernels.call(name + "_forward", *args)
    if impl == "mine":
        sys.path.insert(0, str(ROOT / "tests"))
        import conftest  # noqa: F401  (loads the package)
        from llm_inference_b200 import _lib
        return lambda name, *args: _lib.call("q3_" + name + "_forward", *args)
    raise ValueError(impl)


def run_gpu(impl: str, kind: str, p: dict, inp: dict) -> dict:
    import torch
    L = _launcher(impl)
    s = torch.cuda.current_stream().cuda_stream
    d = {k: _dev(v) for k, v in inp.items()}
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    bf = torch.bfloat16
    if kind == "embedding":
        out = torch.empty(p["hidden"], dtype=bf, device="cuda")
        L("embedding", ptr(out), ptr(d["table"]), ptr(d["token"]), p["hidden"], s)
        res = {"out": out}
    elif kind == "rmsnorm":
        out = torch.empty_like(d["x"])
        L("rmsnorm", ptr(out), ptr(d["x"]), ptr(d["w"]), p["rows"], p["dim"], 1e-6, s)
        res = {"out": out}
    elif kind == "gemv":
        out = torch.empty(p["rows"], dtype=bf, device="cuda")
        L("gemv", ptr(out), ptr(d["w"]), ptr(d["x"]), p["rows"], p["cols"], s)
        res = {"out": out}
    elif kind == "gemv_residual":
        tap = torch.empty(p["rows"], dtype=bf, device="cuda")
        L("gemv_residual", ptr(d["x"]), ptr(d["w"]), ptr(d["inp"]), p["rows"], p["cols"], ptr(tap), s)
        res = {"x": d["x"], "tap": tap}
    elif kind == "qkv":
        q = torch.empty(p["q_rows"], dtype=bf, device="cuda")
        k = torch.empty(p["kv_rows"], dtype=bf, device="cuda")
        v = torch.empty(p["kv_rows"], dtype=bf, device="cuda")
        L("qkv", ptr(q), ptr(k), ptr(v), ptr(d["wq"]), ptr(d["wk"]), ptr(d["wv"]), ptr(d["x"]),
          p["q_rows"], p["kv_rows"], p["cols"], s)
        res = {"q": q, "k": k, "v": v}
    elif kind == "gate_up":
        act = torch.empty(p["rows"], dtype=bf, device="cuda")
        g = torch.empty_like(act)
        u = torch.empty_like(act)
        L("gate_up", ptr(act), ptr(d["wg"]), ptr(d["wu"]), ptr(d["x"]), p["rows"], p["cols"], ptr(g), ptr(u), s)
        res = {"act": act, "gate": g, "up": u}
    elif kind == "qk_norm_rope":
        kvd = p["n_kv"] * p["hd"]
        kc = torch.zeros(p["max_seq"], kvd, dtype=bf, device="cuda")
        vc = torch.zeros_like(kc)
        qt = torch.empty_like(d["q"])
        kt = torch.empty_like(d["k"])
        L("qk_norm_rope", ptr(d["q"]), ptr(d["k"]), ptr(d["v"]), ptr(d["qn"]), ptr(d["kn"]), ptr(kc), ptr(vc),
          ptr(d["pos"]), p["n_heads"], p["n_kv"], p["hd"], 1e-6, 1e6, ptr(qt), ptr(kt), s)
        torch.cuda.synchronize()
        others = torch.cat([kc[:p["pos"]], kc[p["pos"] + 1:], vc[:p["pos"]], vc[p["pos"] + 1:]])
        assert not others.view(torch.int16).any(), "qk_norm_rope wrote outside cache row pos"
        res = {"q": d["q"], "k": d["k"], "q_tap": qt, "k_tap": kt, "krow": kc[p["pos"]], "vrow": vc[p["pos"]]}
    elif kind == "attention":
        out = torch.empty(p["n_heads"] * p["hd"], dtype=bf, device="cuda")
        att = torch.empty(p["n_heads"] * p["max_seq"], dtype=torch.float32, device="cuda")
        scale = float(np.float32(1.0 / math.sqrt(p["hd"])))
        L("attention", ptr(out), ptr(d["q"]), ptr(d["kc"]), ptr(d["vc"]), ptr(att), p["n_heads"], p["n_kv"],
          p["hd"], ptr(d["pos"]), p["max_seq"], scale, s)
        res = {"out": out}
    elif kind == "argmax":
        out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
        L("argmax", ptr(out), ptr(d["x"]), p["n"], s)
        res = {"out": out}
    elif kind == "sample":
        out = torch.full((1,), -7, dtype=torch.int32, device="cuda")
        L("sample", ptr(out), ptr(d["x"]), p["n"], p["inv_temp"], p["u"], s)
        res = {"out": out}
    else:
        raise ValueError(kind)
    torch.cuda.synchronize()
    return {k: _host(v) for k, v in res.items()}


def run(impl: str, kind: str, p: dict, inp: dict) -> dict:
    return run_oracle(kind, p, inp) if impl == "oracle" else run_gpu(impl, kind, p, inp)


def input_digest(inp: dict) -> str:
    import hashlib
    h = hashlib.sha256()
    for k in sorted(inp):
        h.update(k.encode())
        h.update(np.ascontiguousarray(inp[k]).tobytes())
    return h.hexdigest()[:16]
