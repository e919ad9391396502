"""Batched kernels on a B200 against the batch-1 kernels applied sequence by sequence.

The batch-1 launchers are bit-identical to the reference kernels (test_kernels_gpu.py), so
running them once per sequence gives the reference's answer for the batch. The batched
projections (tcgen05, B >= 2) and the split-KV attention sum in a different fp32 order; their
bar is tests/parity.check_close:
  - at most 1 bf16 ulp for all but 0.5% of elements, and
  - every element within |mine - ref| <= 2^-7 * |ref| + 2^-17 * sum_k |terms_k| (fp32
    reordering error is bounded by the sum of absolute terms; near-zero results can move by
    more than one ulp, never by more than that bound). For the residual x = bf16(x0 + y) the
    bound adds y's own bound, 2^-7 * |y|: one ulp of y survives the add even when x0 + y
    cancels to a small x. For attention the sum of absolute terms is sum_t p_t |v_t|, computed
    per output element.
The batched SwiGLU output is checked on every element: it must be the reference's SwiGLU
(src/kernels.cu:277-286) of the batched kernel's own gate and up values, and those are within
the bar above. Gathers, positions and argmax are checked bit for bit. Every comparison's
maximum ulp distance is recorded and printed at the end of the run (conftest.py).
"""
import math
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE / "golden"))
import conftest  # noqa: E402,F401
import oracle as O  # noqa: E402
from parity import attention_abs_terms, bits, check_close, check_ulp, swiglu_of  # noqa: E402,F401

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import llm_inference_b200 as q3  # noqa: E402
from llm_inference_b200 import _lib  # noqa: E402


def rn(g, *shape, std=1.0, mean=0.0):
    return (torch.randn(*shape, generator=g, device="cuda") * std + mean).bfloat16()


def stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("batch", [2, 16, 32, 64, 256])
@pytest.mark.parametrize("rows,cols", [(2560, 4096), (6144, 2560), (100, 72), (1000, 9728)])
def test_batched_gemv_residual_matches_per_sequence(batch, rows, cols):
    g = torch.Generator(device="cuda").manual_seed(batch * 7 + rows)
    w = rn(g, rows, cols, std=0.02)
    inp = rn(g, batch, cols)
    x0 = rn(g, batch, rows)
    x = x0.clone()
    tap = torch.empty(batch, rows, dtype=torch.bfloat16, device="cuda")
    _lib.call("q3_gemv_residual_batched", x.data_ptr(), w.data_ptr(), inp.data_ptr(), batch, rows, cols,
              tap.data_ptr(), stream())
    ref_x = x0.clone()
    ref_tap = torch.empty_like(tap)
    for b in range(batch):
        q3.gemv_residual_forward(ref_x[b], w, inp[b], rows, cols, tap=ref_tap[b])
    absw = (w.float().abs() @ inp.float().abs().T).T  # [batch, rows] sum of |terms|
    torch.cuda.synchronize()
    check_close(tap, ref_tap, absw, "tap")
    expect_x = (x0.float() + tap.float()).bfloat16()
    assert torch.equal(x, expect_x), f"x != bf16(x0 + tap) at {int((x != expect_x).sum())} elements"
    y_bound = np.abs(O.bf16_to_f32(bits(ref_tap))) * 2.0 ** -7
    check_close(x, ref_x, absw, "x", extra=y_bound)
    assert q3.device_error() == 0


@pytest.mark.parametrize("batch", [2, 32])
def test_batched_gate_up_qkv_lm_head(batch):
    g = torch.Generator(device="cuda").manual_seed(batch)
    H, I, Q, KV, V = 2560, 9728, 4096, 1024, 151936
    x = rn(g, batch, H)
    wg, wu = rn(g, I, H, std=0.02), rn(g, I, H, std=0.02)
    act = torch.empty(batch, I, dtype=torch.bfloat16, device="cuda")
    gt, ut = torch.empty_like(act), torch.empty_like(act)
    _lib.call("q3_gate_up_batched", act.data_ptr(), wg.data_ptr(), wu.data_ptr(), x.data_ptr(), batch, I, H,
              gt.data_ptr(), ut.data_ptr(), stream())
    r_act, r_g, r_u = torch.empty_like(act), torch.empty_like(act), torch.empty_like(act)
    for b in range(batch):
        q3.gate_up_forward(r_act[b], wg, wu, x[b], I, H, gate_tap=r_g[b], up_tap=r_u[b])
    check_close(gt, r_g, (wg.float().abs() @ x.float().abs().T).T, "gate")
    check_close(ut, r_u, (wu.float().abs() @ x.float().abs().T).T, "up")
    # act, every element: the reference's SwiGLU of the batched kernel's own gate and up (which are
    # within the bar above); host expf may differ from CUDA's in the last fp32 bit, so at most 1 ulp
    check_ulp(act, swiglu_of(bits(gt), bits(ut)).reshape(act.shape), f"act = SwiGLU(gate, up), B={batch}", 1)
    # and the batched act against the reference's act directly, for the record (the propagated gate/up
    # error: SwiGLU's slope is at most about 1.1 |u| in g and |silu(g)| in u)
    gf, uf = gt.float(), ut.float()
    absb = (1.1 * uf.abs() * (wg.float().abs() @ x.float().abs().T).T
            + (gf * torch.sigmoid(gf)).abs() * (wu.float().abs() @ x.float().abs().T).T)
    extra = (2.0 ** -7) * (1.1 * uf.abs() * r_g.float().abs() + (gf * torch.sigmoid(gf)).abs() * r_u.float().abs())
    check_close(act, r_act, absb, f"act vs reference act, B={batch}", extra=extra.cpu().numpy())

    wq, wk, wv = rn(g, Q, H, std=0.02), rn(g, KV, H, std=0.02), rn(g, KV, H, std=0.02)
    q = torch.empty(batch, Q, dtype=torch.bfloat16, device="cuda")
    k, v = torch.empty(batch, KV, dtype=torch.bfloat16, device="cuda"), torch.empty(batch, KV, dtype=torch.bfloat16, device="cuda")
    _lib.call("q3_qkv_batched", q.data_ptr(), k.data_ptr(), v.data_ptr(), wq.data_ptr(), wk.data_ptr(), wv.data_ptr(),
              x.data_ptr(), batch, Q, KV, H, stream())
    rq, rk, rv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    for b in range(batch):
        q3.qkv_forward(rq[b], rk[b], rv[b], wq, wk, wv, x[b], Q, KV, H)
    for mine, ref, w, name in ((q, rq, wq, "q"), (k, rk, wk, "k"), (v, rv, wv, "v")):
        check_close(mine, ref, (w.float().abs() @ x.float().abs().T).T, name)

    emb = rn(g, V, H)
    logits = torch.empty(batch, V, dtype=torch.bfloat16, device="cuda")
    _lib.call("q3_gemv_batched", logits.data_ptr(), emb.data_ptr(), x.data_ptr(), batch, V, H, stream())
    ref = torch.empty_like(logits)
    for b in range(batch):
        q3.gemv_forward(ref[b], emb, x[b], V, H)
    check_close(logits, ref, (emb.float().abs() @ x.float().abs().T).T, "logits")
    best = torch.empty(batch, dtype=torch.int32, device="cuda")
    _lib.call("q3_argmax_batched", best.data_ptr(), logits.data_ptr(), batch, V, stream())
    for b in range(batch):
        assert int(best[b]) == O.argmax(bits(logits[b]))
    assert q3.device_error() == 0


def cache_strides(layout, max_seq, n_kv, hd):
    """(seq, pos, head) element strides of a [B][max_seq][n_kv*hd] ("ref") or [B][n_kv][max_seq][hd]
    ("head") cache."""
    if layout == "ref":
        return max_seq * n_kv * hd, n_kv * hd, hd
    return n_kv * max_seq * hd, hd, max_seq * hd


def to_layout(cache, layout, n_kv, hd):
    """A [B][max_seq][n_kv*hd] cache re-laid out as `layout` (a copy)."""
    if layout == "ref":
        return cache.clone()
    b, t, _ = cache.shape
    return cache.view(b, t, n_kv, hd).permute(0, 2, 1, 3).contiguous()


@pytest.mark.parametrize("layout", ["ref", "head"])
@pytest.mark.parametrize("batch,n_heads,n_kv,hd", [(4, 32, 8, 128), (3, 16, 8, 128), (2, 4, 2, 64)])
def test_batched_rope_and_split_attention(batch, n_heads, n_kv, hd, layout):
    g = torch.Generator(device="cuda").manual_seed(batch + n_heads)
    max_seq = 2600
    kvd = n_kv * hd
    positions = [0, 511, 512, 2599, 1000, 77][:batch]
    kc = rn(g, batch, max_seq, kvd)
    vc = rn(g, batch, max_seq, kvd)
    q = rn(g, batch, n_heads * hd)
    k = rn(g, batch, kvd)
    v = rn(g, batch, kvd)
    qn, kn = rn(g, hd, std=0.02, mean=1.0), rn(g, hd, std=0.02, mean=1.0)
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    strides = cache_strides(layout, max_seq, n_kv, hd)
    # batched rope writes row pos[b] of each sequence's cache; check against per-sequence drop-in
    # calls on the reference layout, then compare in the tested layout
    kc2, vc2, q2, k2 = kc.clone(), vc.clone(), q.clone(), k.clone()
    kl, vl = to_layout(kc, layout, n_kv, hd), to_layout(vc, layout, n_kv, hd)
    _lib.call("q3_qk_norm_rope_batched", q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr(), kn.data_ptr(),
              kl.data_ptr(), vl.data_ptr(), *strides, pos.data_ptr(), batch, n_heads, n_kv, hd, max_seq, 1e-6,
              1e6, None, None, stream())
    for b in range(batch):
        q3.qk_norm_rope_forward(q2[b], k2[b], v[b], qn, kn, kc2[b], vc2[b], pos[b:b + 1], n_heads, n_kv, hd, 1e-6, 1e6)
    assert torch.equal(q, q2) and torch.equal(k, k2)
    assert torch.equal(kl, to_layout(kc2, layout, n_kv, hd)) and torch.equal(vl, to_layout(vc2, layout, n_kv, hd))
    kc, vc = kc2, vc2
    # rows past each sequence's position are never read by the reference: poison them
    for b, p in enumerate(positions):
        kc[b, p + 1:] = float("nan")
        vc[b, p + 1:] = float("nan")
    kl, vl = to_layout(kc, layout, n_kv, hd), to_layout(vc, layout, n_kv, hd)

    scale = float(np.float32(1.0 / math.sqrt(hd)))
    out = torch.empty(batch, n_heads * hd, dtype=torch.bfloat16, device="cuda")
    nbytes = _lib.load().q3_attention_scratch_bytes(batch, n_heads, n_kv, hd, max_seq)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    for rep in range(2):  # the scratch counters must come back to zero: run twice
        _lib.call("q3_attention_batched", out.data_ptr(), q.data_ptr(), kl.data_ptr(), vl.data_ptr(), *strides,
                  scratch.data_ptr(), pos.data_ptr(), batch, n_heads, n_kv, hd, max_seq, scale, stream())
        ref = torch.empty_like(out)
        att = torch.empty(n_heads * max_seq, dtype=torch.float32, device="cuda")
        for b in range(batch):
            q3.attention_forward(ref[b], q[b], kc[b], vc[b], att, n_heads, n_kv, hd, pos[b:b + 1], max_seq, scale)
        absv = attention_abs_terms(q, kc, vc, positions, n_heads, n_kv, hd, scale)
        check_close(out, ref, absv, f"split attention B={batch} {n_heads}/{n_kv} hd{hd} {layout} rep {rep}")
    assert q3.device_error() == 0


def test_batched_embedding_and_token_range():
    g = torch.Generator(device="cuda").manual_seed(5)
    V, H = 1000, 256
    table = rn(g, V, H)
    toks = torch.tensor([5, 999, 0, 17], dtype=torch.int32, device="cuda")
    out = torch.empty(4, H, dtype=torch.bfloat16, device="cuda")
    _lib.call("q3_embedding_batched", out.data_ptr(), table.data_ptr(), toks.data_ptr(), 4, H, V, stream())
    assert torch.equal(out, table[toks.long()])
    assert q3.device_error() == 0
    bad = torch.tensor([3, 1000], dtype=torch.int32, device="cuda")  # 1000 is out of range
    _lib.call("q3_embedding_batched", out.data_ptr(), table.data_ptr(), bad.data_ptr(), 2, H, V, stream())
    assert torch.equal(out[0], table[3]) and not out[1].view(torch.int16).any()
    assert q3.device_error() == 2  # token-range flag, and no read outside the table


# Rows of one prompt share one cache (sequence stride 0) at consecutive positions: the split
# attention then gives an item 16 / NREP rows, so that one V tile in shared memory serves all of
# them (their query heads side by side as the MMA's 16 columns). Each row must come out exactly as
# when it has a cache of its own: the same probabilities, the same chunks, and the tensor cores
# sum each column on its own. Row counts that leave a partial last group, and rows whose ends fall
# in different 512-position chunks.
@pytest.mark.parametrize("rows,n_heads,n_kv,p0", [(7, 32, 8, 3000), (64, 32, 8, 500), (5, 16, 8, 1021),
                                                   (9, 64, 8, 130)])
def test_prompt_rows_sharing_one_cache_match_separate_caches(rows, n_heads, n_kv, p0):
    hd, max_seq = 128, 4096
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + n_heads + p0)
    kvd = n_kv * hd
    kc1 = rn(g, max_seq, kvd)  # [pos][kv heads * hd]: the reference layout, one cache
    vc1 = rn(g, max_seq, kvd)
    q = rn(g, rows, n_heads * hd)
    positions = [p0 + i for i in range(rows)]
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    scale = float(np.float32(1.0 / math.sqrt(hd)))
    nbytes = _lib.load().q3_attention_scratch_bytes(rows, n_heads, n_kv, hd, max_seq)
    shared = torch.empty(rows, n_heads * hd, dtype=torch.bfloat16, device="cuda")
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("q3_attention_batched", shared.data_ptr(), q.data_ptr(), kc1.data_ptr(), vc1.data_ptr(), 0, kvd, hd,
              scratch.data_ptr(), pos.data_ptr(), rows, n_heads, n_kv, hd, max_seq, scale, stream())
    kc = kc1.unsqueeze(0).repeat(rows, 1, 1).contiguous()  # every row its own copy
    vc = vc1.unsqueeze(0).repeat(rows, 1, 1).contiguous()
    own = torch.empty_like(shared)
    scratch.zero_()
    _lib.call("q3_attention_batched", own.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), max_seq * kvd, kvd,
              hd, scratch.data_ptr(), pos.data_ptr(), rows, n_heads, n_kv, hd, max_seq, scale, stream())
    torch.cuda.synchronize()
    assert torch.equal(shared, own), f"{int((shared != own).sum())} of {shared.numel()} elements differ"
    assert q3.device_error() == 0
