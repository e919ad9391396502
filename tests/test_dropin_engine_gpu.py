"""The drop-in, end to end: the reference's own host program (src/main.cu, forward.cu,
loader.cu, dump.cu, unchanged) linked against libqwen3_b200.so instead of its src/kernels.cu,
against the same program linked with its own kernels (the oracle engine). Both are built from
the reference sources by __graft_entry__.build() (llm-inference_b200/_build/dropin_engine and
oracle/_ref/ref_engine).

On a random-init tiny checkpoint in the reference's layout the two must print identical weight
checksums (--checksums), identical greedy tokens (--max-new, graph mode) and bit-identical
activation dumps of every layer (--dump: 17 tensors per layer plus embed, final_norm, logits).
On a Qwen3-4B-shaped checkpoint both run the reference's --bench protocol and print the same
tokens; their rates are recorded (printed at the end of the run).
"""
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(HERE))
import conftest  # noqa: E402,F401
from llm_inference_b200 import checkpoint  # noqa: E402

pytestmark = pytest.mark.gpu

DROPIN = ROOT / "llm-inference_b200" / "_build" / "dropin_engine"
REF_ENGINE = ROOT / "oracle" / "_ref" / "ref_engine"


@pytest.fixture(scope="module")
def setup():
    if not DROPIN.exists() or not REF_ENGINE.exists():
        pytest.skip("drop-in or reference engine not built (they need the reference sources at build time)")
    d = Path(tempfile.mkdtemp())
    model = checkpoint.write_random_checkpoint(d / "model", "tiny", seed=0)
    rng = np.random.default_rng(7)
    tokens = d / "tokens.txt"
    tokens.write_text(" ".join(map(str, rng.integers(0, 1024, 9))) + "\n")
    return d, model, tokens


def run(binary, *args, timeout=300):
    r = subprocess.run([str(binary), *map(str, args)], capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, f"{binary.name} failed:\n{r.stderr[-2000:]}"
    return r


def test_checksums_identical(setup):
    _, model, _ = setup
    a = run(DROPIN, model, "--checksums").stdout
    b = run(REF_ENGINE, model, "--checksums").stdout
    assert a == b and len(a.splitlines()) == 24


def test_greedy_tokens_identical(setup):
    _, model, tokens = setup
    a = run(DROPIN, model, "--tokens", tokens, "--max-new", 20).stdout.split()
    b = run(REF_ENGINE, model, "--tokens", tokens, "--max-new", 20).stdout.split()
    assert a == b and len(a) >= 1


def test_layer_dumps_bit_identical(setup):
    d, model, tokens = setup
    da, db = d / "dump_dropin", d / "dump_ref"
    run(DROPIN, model, "--tokens", tokens, "--dump", da)
    run(REF_ENGINE, model, "--tokens", tokens, "--dump", db)
    names = sorted(p.name for p in db.glob("*.bin"))
    assert len(names) == 1 + 17 * 2 + 2
    for name in names:
        a = np.fromfile(da / name, dtype=np.float32)
        b = np.fromfile(db / name, dtype=np.float32)
        assert a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32)), name


def _bench(binary, model, tokens, steps, runs):
    r = run(binary, model, "--tokens", tokens, "--bench", steps, "--runs", runs, timeout=900)
    secs = [float(line.split()[3]) for line in r.stdout.splitlines() if line.startswith("run ")]
    assert len(secs) == runs
    return sorted(steps / s for s in secs)[runs // 2]


def test_bench_qwen3_4b_against_reference_kernels(tmp_path):
    """Both programs on a random Qwen3-4B checkpoint written from device weights, --bench 128."""
    if not DROPIN.exists() or not REF_ENGINE.exists():
        pytest.skip("drop-in or reference engine not built")
    torch = pytest.importorskip("torch")
    import parity
    from llm_inference_b200.engine import DeviceWeights
    w = DeviceWeights.random(checkpoint.PRESETS["qwen3-4b"], seed=0)
    torch.cuda.synchronize()
    model = w.save(tmp_path / "model4b")
    del w
    torch.cuda.empty_cache()
    tokens = tmp_path / "tokens.txt"
    tokens.write_text("17\n")
    mine = _bench(DROPIN, model, tokens, 128, 3)
    ref = _bench(REF_ENGINE, model, tokens, 128, 3)
    parity.MEASURES.append(f"drop-in --bench 128 at Qwen3-4B: this library {mine:.1f} tok/s, "
                           f"reference kernels {ref:.1f} tok/s ({mine / ref:.2f}x)")
    a = run(DROPIN, model, "--tokens", tokens, "--max-new", 8, timeout=900).stdout.split()
    b = run(REF_ENGINE, model, "--tokens", tokens, "--max-new", 8, timeout=900).stdout.split()
    assert a == b


def test_bench_mode_runs(setup):
    _, model, tokens = setup
    out = run(DROPIN, model, "--tokens", tokens, "--bench", 16, "--runs", 2).stdout
    assert sum(1 for line in out.splitlines() if line.startswith("run ")) == 2
