"""q3_rope_attention_batched (RoPE + attention in one launch) on a B200 against the bit-exact
kernels: the drop-in qk_norm_rope_forward (bit-identical to the reference's qk_norm_rope) followed
by the drop-in attention_forward (bit-identical to the reference's attention) per sequence.

  - the new key and value rows land in the caches bit for bit, and nothing else changes there
    or in q, k, v;
  - with one chunk the output is the reference's bit for bit;
  - with the chunk count that fills the GPU, only the fp32 order of the P.V sum differs: the
    split-attention bar of tests/parity.check_close applies (at most 1 bf16 ulp for all but
    0.5 % of elements, every element within 2^-7 |ref| + 2^-17 sum_t p_t |v_t|);
  - every case runs twice, and cache rows past each position hold NaN, which must never be read.
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

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import llm_inference_b200 as q3  # noqa: E402
from llm_inference_b200 import _lib  # noqa: E402
from parity import attention_abs_terms, check_close  # noqa: E402
from test_batched_gpu import cache_strides, rn, stream, to_layout  # noqa: E402

EPS, THETA = 1e-6, 1e6


def reference(q, k, v, qn, kn, kc, vc, pos, n_heads, n_kv, hd, max_seq, scale):
    """Caches [B][max_seq][n_kv*hd] after the exact RoPE kernel, and the exact attention output."""
    batch = q.shape[0]
    q2, k2, kc2, vc2 = q.clone(), k.clone(), kc.clone(), vc.clone()
    for b in range(batch):
        q3.qk_norm_rope_forward(q2[b], k2[b], v[b], qn, kn, kc2[b], vc2[b], pos[b:b + 1], n_heads, n_kv, hd, EPS,
                                THETA)
    out = torch.empty_like(q)
    att = torch.empty(n_heads * max_seq, dtype=torch.float32, device="cuda")
    for b in range(batch):
        q3.attention_forward(out[b], q2[b], kc2[b], vc2[b], att, n_heads, n_kv, hd, pos[b:b + 1], max_seq, scale)
    return kc2, vc2, out, q2


CASES = [  # batch, n_heads, n_kv, hd, positions
    (1, 32, 8, 128, [2047]),
    (1, 32, 8, 128, [0]),
    (1, 16, 8, 128, [130]),
    (2, 4, 2, 64, [255, 1]),
    (4, 32, 8, 128, [0, 511, 2599, 77]),
    (3, 8, 1, 128, [128, 129, 1000]),
    (2, 64, 8, 128, [300, 2000]),
]


@pytest.mark.parametrize("layout", ["ref", "head"])
@pytest.mark.parametrize("batch,n_heads,n_kv,hd,positions", CASES)
def test_rope_attention_matches_exact_kernels(batch, n_heads, n_kv, hd, positions, layout):
    lib = _lib.load()
    max_seq = 2600
    auto = lib.q3_rope_attention_chunks(batch, n_heads, n_kv, hd, max_seq)
    assert auto >= 2, "the fused kernel should apply to these shapes"
    g = torch.Generator(device="cuda").manual_seed(batch * 31 + n_heads + hd)
    kvd = n_kv * hd
    kc = rn(g, batch, max_seq, kvd)
    vc = rn(g, batch, max_seq, kvd)
    for b, p in enumerate(positions):  # rows past each position are never read: poison them
        kc[b, p + 1:] = float("nan")
        vc[b, p + 1:] = float("nan")
    q = rn(g, batch, n_heads * hd)
    k = rn(g, batch, kvd)
    v = rn(g, batch, kvd)
    qn, kn = rn(g, hd, std=0.02, mean=1.0), rn(g, hd, std=0.02, mean=1.0)
    pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
    scale = float(np.float32(1.0 / math.sqrt(hd)))
    ref_kc, ref_vc, ref_out, q_rope = reference(q, k, v, qn, kn, kc, vc, pos, n_heads, n_kv, hd, max_seq, scale)
    absv = attention_abs_terms(q_rope, ref_kc, ref_vc, positions, n_heads, n_kv, hd, scale)
    strides = cache_strides(layout, max_seq, n_kv, hd)
    q0, k0, v0 = q.clone(), k.clone(), v.clone()
    # one chunk holds every position's scores in shared memory: too many at 8 query heads per kv
    # head and 2600 positions, which the call refuses
    one = [1] if n_heads // n_kv <= 4 else []
    if not one:
        with pytest.raises(q3.Q3Error) as err:
            _lib.call("q3_rope_attention_batched", q.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr(),
                      kn.data_ptr(), kc.data_ptr(), vc.data_ptr(), *cache_strides("ref", max_seq, n_kv, hd),
                      pos.data_ptr(), batch, n_heads, n_kv, hd, max_seq, EPS, THETA, scale, 1, stream())
        assert err.value.status == 1  # Q3_ERR_SHAPE, and nothing launched
    for chunks in sorted(set(one + [3, auto])):
        for rep in range(2):
            kl, vl = to_layout(kc, layout, n_kv, hd), to_layout(vc, layout, n_kv, hd)
            out = torch.full_like(q, float("nan"))
            _lib.call("q3_rope_attention_batched", out.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                      qn.data_ptr(), kn.data_ptr(), kl.data_ptr(), vl.data_ptr(), *strides, pos.data_ptr(), batch,
                      n_heads, n_kv, hd, max_seq, EPS, THETA, scale, chunks, stream())
            torch.cuda.synchronize()
            assert q3.device_error() == 0
            assert torch.equal(q, q0) and torch.equal(k, k0) and torch.equal(v, v0)
            # caches: bit for bit (NaN rows compared as bits)
            for mine, ref in ((kl, ref_kc), (vl, ref_vc)):
                assert torch.equal(mine.view(torch.int16), to_layout(ref, layout, n_kv, hd).view(torch.int16))
            what = f"chunks {chunks} rep {rep}"
            if chunks == 1:
                assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16)), what
            else:
                check_close(out, ref_out, absv, f"fused attention B={batch} {n_heads}/{n_kv} hd{hd} {layout} {what}")


def test_rope_attention_rejects_bad_arguments():
    lib = _lib.load()
    batch, n_heads, n_kv, hd, max_seq = 2, 32, 8, 128, 256
    auto = lib.q3_rope_attention_chunks(batch, n_heads, n_kv, hd, max_seq)
    assert auto >= 2
    assert lib.q3_rope_attention_chunks(batch, n_heads, n_kv, 96, max_seq) == 0  # head_dim 96: not this kernel
    assert lib.q3_rope_attention_chunks(batch, 24, 8, 128, max_seq) == 0           # group size 3
    assert lib.q3_rope_attention_chunks(4096, n_heads, n_kv, hd, max_seq) == 0     # too many sequences
    assert lib.q3_rope_attention_chunks(1, n_heads, n_kv, hd, 10 ** 7) == 0        # chunk scores too long
    t = torch.zeros(batch * max_seq * n_kv * hd, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(batch, dtype=torch.int32, device="cuda")
    strides = cache_strides("head", max_seq, n_kv, hd)
    args = [t.data_ptr()] * 8 + list(strides) + [pos.data_ptr(), batch, n_heads, n_kv, hd, max_seq, EPS, THETA, 0.1]
    with pytest.raises(q3.Q3Error):  # more chunks than a cluster takes
        _lib.call("q3_rope_attention_batched", *args, 17, stream())
    with pytest.raises(q3.Q3Error):  # sequences sharing one cache
        _lib.call("q3_rope_attention_batched", *args[:8], 0, *strides[1:], *args[11:], auto, stream())
    with pytest.raises(q3.Q3Error):  # no output
        _lib.call("q3_rope_attention_batched", None, *args[1:], auto, stream())
    torch.cuda.synchronize()
    assert q3.device_error() == 0
