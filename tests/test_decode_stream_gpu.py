"""The batch-1 streaming decode kernel (Q3_ENGINE_MEGAKERNEL, csrc/decode_stream.cu) on a B200.

One cooperative launch per token runs the whole decode step, its weights streamed through a
shared-memory ring by a producer warp per SM. Its arithmetic is the reference's everywhere except
the order of the P.V sums (chunk partials added in chunk order), so:
  - greedy tokens equal the CPU oracle's wherever its top-2 logit gap exceeds 1e-2;
  - every step's logits stay within a few bf16 ulps of the batch-1 engine with exact attention,
    teacher-forced on the same tokens, over prompts long enough for many chunks per kv head;
  - the K and V rows of position 0 land in the cache bit for bit as the exact engine writes them;
  - steps replayed on the device (q3_engine_step) give the same tokens as the per-token protocol;
  - shapes it cannot run are refused at engine creation.
"""
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE / "golden"))
import conftest  # noqa: E402,F401
import oracle as O  # noqa: E402
from parity import bits, record  # noqa: E402

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import llm_inference_b200 as q3  # noqa: E402
from llm_inference_b200 import checkpoint  # noqa: E402
from llm_inference_b200.engine import DeviceWeights, Engine  # noqa: E402

# head_dim 128 (the kernel's), GQA 2, small enough for the CPU oracle
HD128 = checkpoint.Qwen3Shape(256, 512, 2, 4, 2, 128, 1024, max_position_embeddings=4096, eos_token_id=[1023])
# GQA 4 and 8, odd row counts against the 148 CTAs
GQA4 = checkpoint.Qwen3Shape(512, 1536, 2, 8, 2, 128, 3001, max_position_embeddings=4096, eos_token_id=[1])
GQA8 = checkpoint.Qwen3Shape(384, 1024, 3, 8, 1, 128, 2000, max_position_embeddings=4096, eos_token_id=[1])


def decode(eng, prompt, n_new):
    logits = []
    for p, t in enumerate(prompt):
        eng.forward([t], [p])
        logits.append(eng.logits()[0].float().cpu().clone())
    toks = [eng.sample_argmax()[0]]
    for i in range(1, n_new):
        eng.forward([toks[-1]], [len(prompt) + i - 1])
        logits.append(eng.logits()[0].float().cpu().clone())
        toks.append(eng.sample_argmax()[0])
    return toks, logits


def test_stream_tokens_match_oracle():
    d = checkpoint.write_random_checkpoint(tempfile.mkdtemp(), HD128, seed=0)
    cfg, tensors = O.load_model(d)
    w = DeviceWeights.from_checkpoint(d)
    eng = Engine(w, batch=1, max_seq=64, megakernel=True)
    prompt = np.random.default_rng(123).integers(0, cfg["vocab_size"], 6).tolist()
    toks, _ = decode(eng, prompt, 12)
    m = O.OracleModel(cfg, tensors, max_seq=64)
    ref_toks, ref_logits = m.greedy(prompt, 12)
    for i, (a, r) in enumerate(zip(toks, ref_toks)):
        if a != r:
            f = np.sort(O.bf16_to_f32(ref_logits[len(prompt) - 1 + i]))[::-1]
            assert f[0] - f[1] <= 1e-2, f"step {i}: {a} vs oracle {r}"
            break
    eng.close()
    assert q3.device_error() == 0


@pytest.mark.parametrize("shape_name", ["hd128", "gqa4", "gqa8"])
def test_stream_logits_close_to_exact_engine(shape_name):
    shape = {"hd128": HD128, "gqa4": GQA4, "gqa8": GQA8}[shape_name]
    w = DeviceWeights.random(shape, seed=7)
    rng = np.random.default_rng(8)
    prompt = rng.integers(0, shape.vocab_size, 700).tolist()  # many chunks per kv head
    ref = Engine(w, batch=1, max_seq=1024, exact_attention=True)
    mk = Engine(w, batch=1, max_seq=1024, megakernel=True)
    worst = 0
    # the same tokens through both (teacher forcing), so every step compares like with like
    for p, t in enumerate(prompt):
        ref.forward([t], [p])
        mk.forward([t], [p])
        if p % 37 == 0 or p == len(prompt) - 1:
            a, b = mk.logits()[0], ref.logits()[0]
            d = O.ulp_diff(bits(a), bits(b))
            worst = max(worst, int(d.max()))
            af, bf = a.float(), b.float()
            err = (af - bf).abs()
            bound = 2.0 ** -5 * bf.abs() + 2.0 ** -6
            assert bool((err <= bound).all()), f"position {p}: max error {err.max().item():.4g}"
            if p == 0:  # one position: P.V is one product per chunk, the logits are exact
                assert torch.equal(a, b)
    record(f"streaming kernel vs exact engine logits, {shape_name}, positions 0..699", np.array([worst]), 1,
           "within 2^-5 |ref| + 2^-6 (P.V order only)")
    # the caches the two engines wrote: position 0 bit for bit (nothing before it differs); later
    # rows carry the P.V-order differences of the layers below (the logits bar covers them)
    L, kv, hd = shape.num_hidden_layers, shape.num_key_value_heads, shape.head_dim
    for buf in ("key_cache", "value_cache"):
        x = q3.engine.device_view(getattr(mk.info, buf), (L, 1, kv, 1024, hd), "bf16")
        y = q3.engine.device_view(getattr(ref.info, buf), (L, 1, kv, 1024, hd), "bf16")
        assert torch.equal(x[:, :, :, 0], y[:, :, :, 0]), buf
    ref.close()
    mk.close()
    assert q3.device_error() == 0


def test_stream_device_loop_matches_protocol():
    shape = GQA4
    w = DeviceWeights.random(shape, seed=9)
    prompt = np.random.default_rng(10).integers(0, shape.vocab_size, 5).tolist()
    a = Engine(w, batch=1, max_seq=64, megakernel=True)
    toks, _ = decode(a, prompt, 8)
    a.close()
    b = Engine(w, batch=1, max_seq=64, megakernel=True, history_cap=32)
    for p, t in enumerate(prompt):
        b.forward([t], [p])
    b.capture()
    b.step(7)
    torch.cuda.synchronize()
    hist = b.history().cpu().numpy()[:, 0].tolist()
    assert hist[len(prompt) - 1:len(prompt) - 1 + 8] == toks
    assert b.positions().cpu().tolist() == [len(prompt) + 7]
    assert b.launches_per_step() == 1
    b.close()
    assert q3.device_error() == 0


def test_stream_refuses_unsupported_shapes():
    w = DeviceWeights.random(checkpoint.PRESETS["tiny"], seed=1)  # head_dim 64
    with pytest.raises(q3.Q3Error):
        Engine(w, batch=1, max_seq=32, megakernel=True)
    w = DeviceWeights.random(HD128, seed=1)
    with pytest.raises(q3.Q3Error):
        Engine(w, batch=2, max_seq=32, megakernel=True)
