"""The decode engine (csrc/engine.cu) on a B200 against the CPU oracle's forward pass.

A random-init tiny Qwen3 checkpoint (the reference's on-disk layout) is decoded greedily:
prompt positions one at a time, then generated tokens, as the reference's main.cu does.
  - batch 1 with the bit-exact attention: every step's logits equal the oracle's bit for bit
    and the tokens are identical;
  - batch 1 and 4 with split-KV attention (and tcgen05 projections at batch 4): tokens are
    identical to the oracle's wherever the oracle's top-2 logit gap exceeds 1e-2; a flip at a
    closer gap ends that sequence's comparison;
  - the captured, device-resident loop produces the same tokens as the per-token protocol.
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

N_PROMPT, N_NEW = 6, 12


@pytest.fixture(scope="module")
def model():
    d = checkpoint.write_random_checkpoint(tempfile.mkdtemp(), "tiny", seed=0)
    cfg, tensors = O.load_model(d)
    return d, cfg, tensors


def prompts(batch, vocab):
    rng = np.random.default_rng(123)
    return rng.integers(0, vocab, (batch, N_PROMPT)).tolist()


def oracle_decode(cfg, tensors, prompt):
    m = O.OracleModel(cfg, tensors, max_seq=64)
    toks, logits = m.greedy(prompt, N_NEW)
    gaps = []
    for lg in logits[N_PROMPT - 1:]:
        f = np.sort(O.bf16_to_f32(lg))[::-1]
        gaps.append(float(f[0] - f[1]))
    return toks, logits, gaps


def engine_decode(eng, prompt_batch):
    B = len(prompt_batch)
    logits = []
    for p in range(N_PROMPT):
        eng.forward([pr[p] for pr in prompt_batch], [p] * B)
        logits.append(eng.logits().clone())
    toks = [eng.sample_argmax()]
    for i in range(1, N_NEW):
        eng.forward(toks[-1], [N_PROMPT + i - 1] * B)
        logits.append(eng.logits().clone())
        toks.append(eng.sample_argmax())
    return np.array(toks).T.tolist(), logits


def bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_batch1_exact_attention_is_bit_exact(model):
    d, cfg, tensors = model
    w = DeviceWeights.from_checkpoint(d)
    eng = Engine(w, batch=1, max_seq=64, exact_attention=True)
    pr = prompts(1, cfg["vocab_size"])
    toks, logits = engine_decode(eng, pr)
    ref_toks, ref_logits, _ = oracle_decode(cfg, tensors, pr[0])
    assert toks[0] == ref_toks
    for step, (a, b) in enumerate(zip(logits, ref_logits)):
        assert np.array_equal(bits(a[0]), b), f"logits differ at step {step}"
    eng.close()
    assert q3.device_error() == 0


@pytest.mark.parametrize("batch", [1, 4])
def test_split_attention_and_batched_tokens(model, batch):
    d, cfg, tensors = model
    w = DeviceWeights.from_checkpoint(d)
    eng = Engine(w, batch=batch, max_seq=64)
    prs = prompts(batch, cfg["vocab_size"])
    toks, _ = engine_decode(eng, prs)
    for b in range(batch):
        ref_toks, _, gaps = oracle_decode(cfg, tensors, prs[b])
        for i, (a, r) in enumerate(zip(toks[b], ref_toks)):
            if a != r:
                assert gaps[i] <= 1e-2, f"sequence {b} step {i}: {a} vs oracle {r}, gap {gaps[i]:.4f}"
                break
    eng.close()
    assert q3.device_error() == 0


def test_device_loop_matches_protocol(model):
    d, cfg, _ = model
    w = DeviceWeights.from_checkpoint(d)
    batch = 3
    prs = prompts(batch, cfg["vocab_size"])
    eng = Engine(w, batch=batch, max_seq=64)
    toks, _ = engine_decode(eng, prs)
    eng.close()

    loop = Engine(w, batch=batch, max_seq=64, history_cap=64)
    for p in range(N_PROMPT):
        loop.forward([pr[p] for pr in prs], [p] * batch)
    loop.capture()
    loop.step(N_NEW - 1)
    torch.cuda.synchronize()
    hist = loop.history().cpu().numpy()
    got = hist[N_PROMPT - 1:N_PROMPT - 1 + N_NEW].T.tolist()
    assert got == toks
    assert loop.positions().cpu().tolist() == [N_PROMPT + N_NEW - 1] * batch
    loop.close()
    assert q3.device_error() == 0


def test_engine_switches_to_split_attention_at_long_context():
    """A batch-1 engine runs the fused RoPE + attention launch up to split_from and the split-KV
    kernels from there on, as a second captured graph. Qwen3-4B shapes cut to 2 layers, caches
    filled identically: from split_from on its logits equal those of an engine created with
    split attention throughout, bit for bit (same kernels); below it they agree to the fused
    P.V's reordering; the device loop crosses the switch with positions advancing one a step."""
    full = checkpoint.PRESETS["qwen3-4b"]
    shape = checkpoint.Qwen3Shape(full.hidden_size, full.intermediate_size, 2, full.num_attention_heads,
                                  full.num_key_value_heads, full.head_dim, full.vocab_size)
    max_seq = 8192
    w = DeviceWeights.random(shape, seed=3)
    auto = Engine(w, batch=1, max_seq=max_seq, history_cap=16)
    split = Engine(w, batch=1, max_seq=max_seq, history_cap=16, split_attention=True)
    sf = auto.split_from()
    assert 0 < sf < max_seq, sf
    assert split.split_from() == -1
    for e in (auto, split):
        e.fill_kv_normal(max_seq, seed=29)
        e.capture()
    auto.forward([321], [sf + 3])
    split.forward([321], [sf + 3])
    torch.cuda.synchronize()
    assert torch.equal(auto.logits().view(torch.int16), split.logits().view(torch.int16))
    assert auto.launches_per_step() == split.launches_per_step()
    auto.forward([321], [sf - 5])
    split.forward([321], [sf - 5])
    torch.cuda.synchronize()
    assert auto.launches_per_step() < split.launches_per_step()  # the fused launch again
    a, s = auto.logits().float(), split.logits().float()
    rel = float(((a - s).pow(2).mean() / s.pow(2).mean()).sqrt())
    assert rel < 1e-2, rel
    auto.set_state([7], [sf - 2])
    auto.step(4)
    torch.cuda.synchronize()
    assert auto.positions().cpu().tolist() == [sf + 2]
    for e in (auto, split):
        e.close()
    assert q3.device_error() == 0
