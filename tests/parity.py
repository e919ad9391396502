"""Parity checks shared by the GPU tests, and the record of what they measured.

``check_close(mine, ref, absbound, what)`` is the bar for paths that sum in a different fp32
order than the reference kernels (tcgen05 projections, split-KV attention):
  - at most 1 bf16 ulp for all but 0.5 % of elements, and
  - every element within |mine - ref| <= 2^-7 * |ref| + 2^-17 * sum_k |terms_k|. The first term
    is one bf16 ulp of the result; the second covers the fp32 reordering error, which for a sum
    of n terms in another order grows like sqrt(n) * 2^-24 * sum |terms| (rounding errors of
    either sign): 2^-17 covers that up to n of about 16k terms. It is a statistical bar, not a
    worst-case bound (n * 2^-24 * sum |terms|). Near-zero results can move by more than one ulp,
    never by more than this bar.
NaN must appear exactly where the reference has NaN.

Every call records the maximum ulp distance, the count of elements more than 1 ulp away and
the count that is not bit-identical; ``conftest.py`` prints the table at the end of the run and,
when the environment variable Q3_PARITY_LOG names a file, writes it there as JSON lines.
"""
from __future__ import annotations

import numpy as np

import oracle as O

RECORDS: list[dict] = []
MEASURES: list[str] = []  # timings some GPU tests take on the way (printed at the end of the run)


def bits(t) -> np.ndarray:
    import torch
    if isinstance(t, np.ndarray):
        return t.view(np.uint16)
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def record(what: str, d: np.ndarray, n: int, bound: str) -> dict:
    r = {"what": what, "elements": int(n), "max_ulp": int(d.max()) if d.size else 0,
         "over_1ulp": int(np.count_nonzero(d > 1)), "not_identical": int(np.count_nonzero(d > 0)), "bar": bound}
    RECORDS.append(r)
    return r


def check_equal(mine, ref, what: str) -> dict:
    """Bit-identical bf16 tensors (NaN payloads included)."""
    m, r = bits(mine).reshape(-1), bits(ref).reshape(-1)
    d = O.ulp_diff(m, r)
    rec = record(what, d, m.size, "bit-identical")
    assert np.array_equal(m, r), f"{what}: {rec['not_identical']} elements differ (max {rec['max_ulp']} ulp)"
    return rec


def check_ulp(mine, ref, what: str, max_ulp: int = 1) -> dict:
    """Every element within `max_ulp` bf16 ulps."""
    m, r = bits(mine).reshape(-1), bits(ref).reshape(-1)
    d = O.ulp_diff(m, r)
    rec = record(what, d, m.size, f"<= {max_ulp} ulp")
    mf, rf = O.bf16_to_f32(m), O.bf16_to_f32(r)
    assert np.array_equal(np.isnan(mf), np.isnan(rf)), f"{what}: NaN pattern differs"
    assert rec["max_ulp"] <= max_ulp, f"{what}: {rec['max_ulp']} ulp at index {int(d.argmax())}"
    return rec


def check_close(mine, ref, absbound, what: str, extra=None) -> dict:
    m, r = bits(mine).reshape(-1), bits(ref).reshape(-1)
    d = O.ulp_diff(m, r)
    rec = record(what, d, m.size, "<= 1 ulp on >= 99.5 %, all within the fp32 reordering bound")
    frac_over = rec["over_1ulp"] / max(1, m.size)
    mf, rf = O.bf16_to_f32(m), O.bf16_to_f32(r)
    if hasattr(absbound, "detach"):
        absbound = absbound.detach().float().cpu().numpy()
    bound = np.abs(rf) * 2.0 ** -7 + np.asarray(absbound, np.float32).reshape(-1) * 2.0 ** -17
    if extra is not None:
        bound = bound + np.asarray(extra, np.float32).reshape(-1)
    assert np.array_equal(np.isnan(mf), np.isnan(rf)), f"{what}: NaN where the reference has none (or the reverse)"
    worst = np.nan_to_num(np.abs(mf - rf) - bound, nan=0.0)
    assert frac_over <= 0.005, f"{what}: {frac_over:.4%} of elements differ by more than 1 ulp (max {d.max()})"
    if worst.max() > 0:
        i = int(worst.argmax())
        bad = int(np.count_nonzero(worst > 0))
        raise AssertionError(f"{what}: error bound exceeded at {bad} elements; first worst index {i} "
                             f"(row-major over {tuple(getattr(mine, 'shape', ()))}): mine {mf[i]} ref {rf[i]} "
                             f"bound {bound[i]}")
    return rec


def swiglu_of(gate_bits: np.ndarray, up_bits: np.ndarray) -> np.ndarray:
    """The reference's SwiGLU epilogue (src/kernels.cu:277-286) applied to given bf16 gate and up
    values: bf16(round_bf16(g / (1 + exp(-g))) * u), in fp32 with the host's expf (the C oracle's
    restatement, qwen3_oracle.c). Host expf and CUDA's may differ in the last fp32 bit, which can
    move a result by one bf16 ulp when it sits on a rounding boundary."""
    g = O.bf16_to_f32(gate_bits).astype(np.float32)
    u = O.bf16_to_f32(up_bits).astype(np.float32)
    with np.errstate(over="ignore"):
        silu = g / (np.float32(1.0) + np.exp(-g, dtype=np.float32))
    silu = O.bf16_to_f32(O.f32_to_bf16(silu.astype(np.float32)))
    return O.f32_to_bf16((silu * u).astype(np.float32))


def attention_abs_terms(q, kc, vc, positions, n_heads: int, n_kv: int, hd: int, scale: float):
    """sum_t p_t * |v_t| per output element of decode attention ([B, n_heads*hd], float32): the
    sum of absolute P.V terms that bounds an fp32 reordering of the P.V sums. q is [B, n_heads*hd];
    kc, vc are [B][max_seq][n_kv*hd] (the reference layout); p is the softmax over 0..pos[b]."""
    import torch
    B = q.shape[0]
    rep = n_heads // n_kv
    out = torch.zeros(B, n_heads * hd, dtype=torch.float32, device=q.device)
    for b, p in enumerate(positions):
        n = int(p) + 1
        k = kc[b, :n].float().view(n, n_kv, hd)
        v = vc[b, :n].float().view(n, n_kv, hd).abs()
        qb = q[b].float().view(n_kv, rep, hd)
        s = torch.einsum("grd,tgd->grt", qb, k) * scale
        pr = torch.softmax(s, dim=-1)
        out[b] = torch.einsum("grt,tgd->grd", pr, v).reshape(-1)
    return out
