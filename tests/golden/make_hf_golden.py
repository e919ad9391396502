"""Generate tests/golden/hf_tiny/: the reference's Hugging Face harness run on a tiny model.

Run in the development container, where the reference tree is mounted (default
$LLM_INFERENCE_REF, else the "reference" directory beside this repository). It imports the reference's own hook set and wiring
check (ref/dump.py: ``install_hooks``, ``check_wiring``) and runs Hugging Face Qwen3 in bf16
with eager attention on the CPU, as ref/calibrate.py does. Outputs:

  hf_tiny/dumps.npz        the 1 + 17 * layers + 2 dumped tensors of a 6-token prompt, as
                           bf16 bits [positions, width], named as the reference dumps them
  hf_tiny/manifest.json    prompt ids, greedy continuation and per-step top-2 logit gaps
                           (the fields ref/dump.py:145-182 records), and the weight checksums
                           of the random-init checkpoint (src/loader.cu:395-419), which the
                           tests regenerate from seed 0 instead of storing it

The tests never import the reference; they read these files.
"""
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "tests"))
import conftest  # noqa: E402  (loads the package)
from llm_inference_b200 import checkpoint  # noqa: E402

REF = Path(os.environ.get("LLM_INFERENCE_REF", str(Path(__file__).resolve().parents[3] / "reference")))
sys.path.insert(0, str(REF / "ref"))
from dump import check_wiring, install_hooks  # noqa: E402  (the reference's harness)

N_PROMPT = 6
N_NEW = 12


def main():
    out = HERE / "hf_tiny"
    out.mkdir(exist_ok=True)
    model_dir = checkpoint.write_random_checkpoint(tempfile.mkdtemp(), "tiny", seed=0)
    _, tensors = checkpoint.read_checkpoint(model_dir)
    sums = {k: list(v) for k, v in checkpoint.weight_checksums(tensors).items()}
    shape = checkpoint.PRESETS["tiny"]

    from transformers import AutoModelForCausalLM
    torch.manual_seed(0)
    model = AutoModelForCausalLM.from_pretrained(model_dir, dtype=torch.bfloat16,
                                                 attn_implementation="eager").eval()
    theta = model.config.rope_parameters["rope_theta"]
    assert theta == shape.rope_theta, theta

    rng = np.random.default_rng(0)
    ids = torch.tensor([rng.integers(0, shape.vocab_size, N_PROMPT).tolist()])
    acts = {}
    remove = install_hooks(model, acts)
    with torch.no_grad():
        model(ids)
    n_layers = shape.num_hidden_layers
    assert len(acts) == 1 + 17 * n_layers + 2, len(acts)
    check_wiring(acts, n_layers, model.model.embed_tokens.weight, ids[0])
    remove()

    arrays = {}
    for name, t in acts.items():
        bits = t.to(torch.bfloat16)
        assert torch.equal(bits.float(), t), f"{name} is not bf16-valued"
        arrays[name] = bits.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(out / "dumps.npz", **arrays)

    with torch.no_grad():
        gen = model.generate(ids, max_new_tokens=N_NEW, do_sample=False, temperature=None,
                             top_p=None, top_k=None, return_dict_in_generate=True,
                             output_logits=True)
    greedy = gen.sequences[0, N_PROMPT:].tolist()
    gaps = []
    for step_logits in gen.logits:
        top2 = step_logits[0].float().topk(2).values
        gaps.append(round(float(top2[0] - top2[1]), 4))
    manifest = {"tokens": ids[0].tolist(), "greedy": greedy, "greedy_top2_gap": gaps,
                "tensors": {k: list(v.shape) for k, v in arrays.items()},
                "preset": "tiny", "seed": 0, "weight_checksums": sums,
                "transformers": __import__("transformers").__version__,
                "torch": torch.__version__}
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1))
    print(f"{len(arrays)} tensors, greedy {greedy}, min gap {min(gaps)}")


if __name__ == "__main__":
    main()
