"""The drop-in, end to end: the reference's own host program (src/main.cu, forward.cu,
loader.cu, dump.cu, unchanged) linked against libqwen3_b200.so instead of its src/kernels.cu,
against the same program linked with its own kernels (the oracle engine). Both are built from
the reference sources by __graft_entry__.build() (llm-inference_b200/_build/dropin_engine and
oracle/_ref/ref_engine).

On a random-init tiny checkpoint in the reference's layout the two must print identical weight
checksums (--checksums), identical greedy tokens (--max-new, graph mode) and bit-identical
activation dumps of every layer (--dump: 17 tensors per layer plus embed, final_norm, logits).
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


def test_bench_mode_runs(setup):
    _, model, tokens = setup
    out = run(DROPIN, model, "--tokens", tokens, "--bench", 16, "--runs", 2).stdout
    assert sum(1 for line in out.splitlines() if line.startswith("run ")) == 2
