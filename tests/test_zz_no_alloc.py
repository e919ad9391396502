"""q3_attention_batched_static: batched attention for callers that cannot allocate device memory.

Some hosts of these kernels cannot call cudaMalloc while they decode: a runtime that reserves all
of its GPU memory in one pool at start-up, a plugin running inside another framework's memory
manager, or a serving loop where an allocation could block or fail in the middle of a request.
For them q3_attention_batched_static takes its scratch from a fixed array inside the library
instead of a caller buffer. These tests call it through the C ABI and compare it with
q3_attention_batched (given a scratch buffer allocated here, in the test) on the same inputs.
Both run the same deterministic kernels, so the outputs must be bit-identical. Two calls in a row
use different positions and queries, so the second one runs over what the first left in the
shared array. A shape that needs more scratch than the array holds must be refused.

The file is named to be collected last: it passes on its own in a fresh process (its first call
does the per-device set-up) and after every other test.
"""
import math
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import conftest  # noqa: E402,F401

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import llm_inference_b200 as q3  # noqa: E402
from llm_inference_b200 import _lib  # noqa: E402
from parity import check_equal  # noqa: E402
from test_batched_gpu import rn, stream  # noqa: E402

STATIC_SCRATCH_BYTES = 32 << 20  # Q3_ATTENTION_STATIC_SCRATCH_BYTES
Q3_ERR_SCRATCH_LIMIT = 6


def head_major(batch, n_kv, max_seq, hd, positions, g):
    """A head-major cache [batch][n_kv][max_seq][hd] of N(0,1) values, NaN past each position."""
    c = rn(g, batch, n_kv, max_seq, hd)
    for b, p in enumerate(positions):
        c[b, :, p + 1:] = float("nan")
    return c


def run_both(q, kc, vc, pos, n_heads, n_kv, hd, max_seq):
    batch = q.shape[0]
    strides = (n_kv * max_seq * hd, hd, max_seq * hd)
    scale = float(np.float32(1.0 / math.sqrt(hd)))
    ref = torch.empty_like(q)
    nbytes = _lib.load().q3_attention_scratch_bytes(batch, n_heads, n_kv, hd, max_seq)
    assert 0 < nbytes <= STATIC_SCRATCH_BYTES
    scratch = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.call("q3_attention_batched", ref.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), *strides,
              scratch.data_ptr(), pos.data_ptr(), batch, n_heads, n_kv, hd, max_seq, scale, stream())
    out = torch.full_like(q, float("nan"))
    _lib.call("q3_attention_batched_static", out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), *strides,
              pos.data_ptr(), batch, n_heads, n_kv, hd, max_seq, scale, stream())
    torch.cuda.synchronize()
    return out, ref


def test_static_scratch_matches_caller_scratch_on_two_calls():
    g = torch.Generator(device="cuda").manual_seed(11)
    n_heads, n_kv, hd, max_seq = 32, 8, 128, 2600
    kc_pos = [2599, 1000, 512, 77]
    kc = head_major(4, n_kv, max_seq, hd, kc_pos, g)
    vc = head_major(4, n_kv, max_seq, hd, kc_pos, g)
    # first call: the longest positions the caches hold; second: shorter ones and other queries,
    # so the array still holds scores and partial sums of the first call beyond the new lengths
    for positions in (kc_pos, [1800, 999, 130, 40]):
        q = rn(g, 4, n_heads * hd)
        pos = torch.tensor(positions, dtype=torch.int32, device="cuda")
        out, ref = run_both(q, kc, vc, pos, n_heads, n_kv, hd, max_seq)
        check_equal(out, ref, f"static scratch, positions {positions}")
    assert q3.device_error() == 0


def test_static_scratch_refuses_shapes_beyond_its_size():
    batch, n_heads, n_kv, hd, max_seq = 32, 32, 8, 128, 8192
    need = _lib.load().q3_attention_scratch_bytes(batch, n_heads, n_kv, hd, max_seq)
    assert need > STATIC_SCRATCH_BYTES
    out = torch.zeros(batch, n_heads * hd, dtype=torch.bfloat16, device="cuda")
    q = torch.zeros_like(out)
    cache = torch.zeros(16, dtype=torch.bfloat16, device="cuda")  # never read: the call is refused first
    pos = torch.zeros(batch, dtype=torch.int32, device="cuda")
    st = _lib.load().q3_attention_batched_static(out.data_ptr(), q.data_ptr(), cache.data_ptr(), cache.data_ptr(),
                                                 n_kv * max_seq * hd, hd, max_seq * hd, pos.data_ptr(), batch,
                                                 n_heads, n_kv, hd, max_seq, 0.088, stream())
    assert st == Q3_ERR_SCRATCH_LIMIT
    assert "scratch" in _lib.load().q3_status_string(st).decode()
    torch.cuda.synchronize()
    assert not out.view(torch.int16).any()
    assert q3.device_error() == 0
