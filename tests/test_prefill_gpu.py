"""Prompt prefill (q3_engine_prefill) against the reference's per-token protocol.

The reference runs a prompt one token per forward (src/main.cu:122-124). The engine's prefill
runs up to `batch` prompt tokens of one sequence per pass: the rows share that sequence's KV
cache at consecutive positions, so each row attends causally.

- **Exact attention, prompt length a multiple of the batch.** Every kernel computes each row
  independently of the other rows, and each pass has the projections' usual shapes. So the
  sequence's cache rows, the last token's logits and the next token must equal, bit for bit,
  those of the per-token protocol run for the same sequence on a second engine.
- **Split-KV attention, head_dim 128 (the tensor-core attention path), ragged last pass, a
  prefill resumed at a non-zero start.** The partial sums of a pass run in another order, so
  the comparison is close, not exact: cache rows and logits within a few bf16 ulps of the
  values, and the same next token wherever the top-2 logit gap exceeds 1e-2.
"""
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
from llm_inference_b200 import checkpoint  # noqa: E402
from llm_inference_b200.engine import DeviceWeights, Engine, device_view  # noqa: E402

SHAPES = {
    "tiny": checkpoint.PRESETS["tiny"],  # head_dim 64
    "hd128": checkpoint.Qwen3Shape(256, 512, 2, 4, 2, 128, 1024, max_position_embeddings=2048, eos_token_id=[1023]),
}
MAX_SEQ = 96
SEQ = 2


def caches(eng, shape):
    """(key, value) caches as [layers, batch, kv heads, max_seq, head_dim] device views."""
    eng.synchronize()
    info = eng.info
    dims = (shape.num_hidden_layers, eng.batch, shape.num_key_value_heads, eng.max_seq, shape.head_dim)
    return device_view(info.key_cache, dims, "bf16"), device_view(info.value_cache, dims, "bf16")


def per_token(eng, prompt, batch, vocab, rng):
    """The reference's protocol for sequence SEQ (the other rows decode unrelated tokens)."""
    for i, t in enumerate(prompt):
        toks = rng.integers(0, vocab, batch).tolist()
        toks[SEQ] = t
        eng.forward(toks, [i] * batch)
    return eng.sample_argmax()[SEQ], eng.logits()[SEQ].clone()


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("name", list(SHAPES))
def test_prefill_matches_per_token_bit_for_bit(name):
    shape = SHAPES[name]
    batch, n = 4, 12
    w = DeviceWeights.random(shape, seed=3)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, shape.vocab_size, n).tolist()

    ref = Engine(w, batch=batch, max_seq=MAX_SEQ, exact_attention=True)
    ref_tok, ref_logits = per_token(ref, prompt, batch, shape.vocab_size, rng)
    ref_k, ref_v = caches(ref, shape)

    eng = Engine(w, batch=batch, max_seq=MAX_SEQ, exact_attention=True)
    eng.prefill(SEQ, prompt)
    tok = eng.sample_argmax()[SEQ]
    logits = eng.logits()[(n - 1) % batch].clone()  # the last pass's last row
    k, v = caches(eng, shape)

    assert tok == ref_tok
    assert np.array_equal(bits(logits), bits(ref_logits))
    assert torch.equal(k[:, SEQ, :, :n], ref_k[:, SEQ, :, :n])
    assert torch.equal(v[:, SEQ, :, :n], ref_v[:, SEQ, :, :n])
    assert eng.positions().cpu().tolist()[SEQ] == n
    # the other sequences' caches were not touched (they start zeroed)
    others = [b for b in range(batch) if b != SEQ]
    assert not k[:, others].view(torch.int16).any() and not v[:, others].view(torch.int16).any()
    ref.close()
    eng.close()
    assert q3.device_error() == 0


def close(a, b, what):
    a, b = a.float(), b.float()
    err = (a - b).abs()
    bound = 2.0 ** -5 * b.abs() + 2.0 ** -6
    assert bool((err <= bound).all()), f"{what}: max error {err.max().item():.4g}"


def test_split_attention_prefill_in_two_calls():
    shape = SHAPES["hd128"]
    batch, n1, n2 = 4, 5, 6  # passes of 4 + 1, then 4 + 2 rows
    w = DeviceWeights.random(shape, seed=4)
    rng = np.random.default_rng(6)
    prompt = rng.integers(0, shape.vocab_size, n1 + n2).tolist()

    ref = Engine(w, batch=batch, max_seq=MAX_SEQ)
    ref_tok, ref_logits = per_token(ref, prompt, batch, shape.vocab_size, rng)
    ref_k, ref_v = caches(ref, shape)

    eng = Engine(w, batch=batch, max_seq=MAX_SEQ)
    eng.prefill(SEQ, prompt[:n1])
    eng.prefill(SEQ, prompt[n1:], start_pos=n1)
    tok = eng.sample_argmax()[SEQ]
    logits = eng.logits()[(n2 - 1) % batch].clone()
    k, v = caches(eng, shape)
    n = n1 + n2

    close(k[:, SEQ, :, :n], ref_k[:, SEQ, :, :n], "key cache")
    close(v[:, SEQ, :, :n], ref_v[:, SEQ, :, :n], "value cache")
    close(logits, ref_logits, "logits")
    top = torch.topk(ref_logits.float(), 2).values
    if float(top[0] - top[1]) > 1e-2:
        assert tok == ref_tok
    assert eng.positions().cpu().tolist()[SEQ] == n
    # decoding continues from the prefilled state on the device loop
    eng.capture()
    eng.step(3)
    assert eng.positions().cpu().tolist()[SEQ] == n + 3
    ref.close()
    eng.close()
    assert q3.device_error() == 0


def test_prefill_rejects_bad_arguments():
    shape = SHAPES["tiny"]
    w = DeviceWeights.random(shape, seed=1)
    eng = Engine(w, batch=2, max_seq=16)
    with pytest.raises(q3.Q3Error):
        eng.prefill(2, [1, 2, 3])          # no such sequence
    with pytest.raises(q3.Q3Error):
        eng.prefill(0, list(range(10)), start_pos=10)  # past max_seq
    with pytest.raises(q3.Q3Error):
        eng.prefill(0, [shape.vocab_size])  # token id out of range
    eng.close()
    assert q3.device_error() == 0


@pytest.mark.parametrize("batch,exact", [(1, True), (4, False)])
def test_prefill_against_oracle_per_token_forward(batch, exact):
    """Prefill against the CPU oracle run the reference's way (one forward per prompt token,
    src/main.cu:122-124, restated in oracle/qwen3_oracle.c). With one-row passes and the exact
    attention every kernel is a bit-exact batch-1 kernel, so the last prompt token's logits equal
    the oracle's bit for bit; with four-row passes (tcgen05 projections, split attention) the
    next token must match wherever the oracle's top-2 gap exceeds 1e-2 and the logits stay close."""
    import tempfile
    sys.path.insert(0, str(HERE / "golden"))
    import oracle as O
    d = checkpoint.write_random_checkpoint(tempfile.mkdtemp(), "tiny", seed=4)
    cfg, tensors = O.load_model(d)
    w = DeviceWeights.from_checkpoint(d)
    prompt = np.random.default_rng(31).integers(0, cfg["vocab_size"], 11).tolist()
    m = O.OracleModel(cfg, tensors, max_seq=MAX_SEQ)
    for p, t in enumerate(prompt):
        ref = m.forward(t, p)
    eng = Engine(w, batch=batch, max_seq=MAX_SEQ, exact_attention=exact)
    seq = batch - 1
    eng.prefill(seq, prompt)
    tok = eng.sample_argmax()[seq]
    # the logits buffer holds the rows of the last pass: the prompt's last token is its last row
    mine = bits(eng.logits()[(len(prompt) - 1) % batch])
    f = np.sort(O.bf16_to_f32(ref))[::-1]
    if exact:
        assert np.array_equal(mine, ref), f"{int((mine != ref).sum())} logits differ from the oracle"
        assert tok == O.argmax(ref)
    else:
        if tok != O.argmax(ref):
            assert f[0] - f[1] <= 1e-2
        mf, rf = O.bf16_to_f32(mine), O.bf16_to_f32(ref)
        assert np.all(np.abs(mf - rf) <= 2.0 ** -5 * np.abs(rf) + 2.0 ** -6)
    assert eng.positions().cpu().tolist()[seq] == len(prompt)
    eng.close()
    assert q3.device_error() == 0
