"""The batch-1 persistent decode kernel (Q3_ENGINE_MEGAKERNEL) on a B200.

One cooperative launch per token runs the whole decode step. Its per-row arithmetic is that of
the batch-1 kernels: exact GEMV order, exact rmsnorm, qk norm and RoPE, exact scores and softmax
statistics. P.V is summed in 128-position parts (64 at head_dim 64). So:
  - greedy tokens equal the CPU oracle's wherever its top-2 logit gap exceeds 1e-2 (the rule of
    the other engine tests);
  - every step's logits stay within a few bf16 ulps of the batch-1 engine with exact attention;
  - steps replayed on the device (q3_engine_step) give the same tokens as the per-token
    protocol;
  - positions past the prompt reach beyond one 256-position item, so the multi-part P.V and
    its combine are covered.
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

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import llm_inference_b200 as q3  # noqa: E402
from llm_inference_b200 import checkpoint  # noqa: E402
from llm_inference_b200.engine import DeviceWeights, Engine  # noqa: E402

HD128 = checkpoint.Qwen3Shape(256, 512, 2, 4, 2, 128, 1024, max_position_embeddings=2048, eos_token_id=[1023])


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


def test_megakernel_tokens_match_oracle():
    d = checkpoint.write_random_checkpoint(tempfile.mkdtemp(), "tiny", seed=0)
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


@pytest.mark.parametrize("shape_name", ["tiny", "hd128"])
def test_megakernel_logits_close_to_batch1_engine(shape_name):
    shape = checkpoint.PRESETS["tiny"] if shape_name == "tiny" else HD128
    w = DeviceWeights.random(shape, seed=7)
    rng = np.random.default_rng(8)
    prompt = rng.integers(0, shape.vocab_size, 300).tolist()  # past one 256-position item
    ref = Engine(w, batch=1, max_seq=512, exact_attention=True)
    mk = Engine(w, batch=1, max_seq=512, megakernel=True)
    # the same tokens through both (teacher forcing), so every step compares like with like
    for p, t in enumerate(prompt):
        ref.forward([t], [p])
        mk.forward([t], [p])
        if p % 37 == 0 or p == len(prompt) - 1:
            a, b = mk.logits()[0].float(), ref.logits()[0].float()
            err = (a - b).abs()
            bound = 2.0 ** -5 * b.abs() + 2.0 ** -6
            assert bool((err <= bound).all()), f"position {p}: max error {err.max().item():.4g}"
    ref.close()
    mk.close()
    assert q3.device_error() == 0


def test_megakernel_device_loop_matches_protocol():
    shape = HD128
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


def test_megakernel_needs_batch_one():
    w = DeviceWeights.random(checkpoint.PRESETS["tiny"], seed=1)
    with pytest.raises(q3.Q3Error):
        Engine(w, batch=2, max_seq=32, megakernel=True)
