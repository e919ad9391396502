"""Generate tests/golden/ref_kernels.npz: outputs of the reference's own CUDA kernels.

Runs on a B200. It needs oracle/_ref/libqwen3_ref.so (the reference's src/kernels.cu compiled
for sm_100a by `make -C oracle ref` in the development container, where the reference tree is
mounted); it does not read the reference sources. For every case of tests/golden/cases.py it
rebuilds the seeded inputs, runs the reference kernel and stores the outputs under
"<case>/<output>", plus "<case>/digest", a hash of the inputs that the tests check so that a
change in input generation cannot pass unnoticed.

    python tests/golden/make_ref_kernel_golden.py [out.npz]
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402


def main():
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE / "ref_kernels.npz"
    import torch
    assert torch.cuda.is_available()
    arrays = {}
    for kind, name, p in cases.CASES:
        inp = cases.inputs(kind, p)
        res = cases.run("ref", kind, p, inp)
        for k, v in res.items():
            arrays[f"{name}/{k}"] = v
        arrays[f"{name}/digest"] = np.array(cases.input_digest(inp))
        print(f"{name}: {', '.join(f'{k}{list(v.shape)}' for k, v in res.items())}", flush=True)
    out.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({out.stat().st_size} bytes, {torch.cuda.get_device_name()})")


if __name__ == "__main__":
    main()
