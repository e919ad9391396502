"""Checkpoint layout and validation (checkpoint.py), the rules of the reference's loader
(src/loader.cu:113-140, :313-380), on CPU; and the fast device loader against the plain one on a
B200.

- A written random checkpoint reads back bit for bit through the header-only layout and the
  memory-mapped reader.
- Each malformed checkpoint raises CheckpointError: missing tensor, wrong dtype, wrong shape,
  misaligned data, an unused tensor, no eos token, a negative or non-integer data offset (which
  would otherwise read the header as weights), and one tensor name in two shards.
"""
import json
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import conftest  # noqa: E402,F401

from llm_inference_b200 import checkpoint as ckpt  # noqa: E402


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    d = tmp_path_factory.mktemp("ckpt")
    ckpt.write_random_checkpoint(d, "tiny", seed=3)
    return d


def test_layout_and_reader_round_trip(tiny):
    shape, spans = ckpt.checkpoint_layout(tiny)
    assert (shape.hidden_size, shape.num_hidden_layers) == (256, 2)
    want = ckpt.random_tensors(ckpt.PRESETS["tiny"], seed=3)
    assert set(spans) == set(want)
    _, tensors = ckpt.read_checkpoint(tiny)
    raw = (tiny / "model.safetensors").read_bytes()
    for name, a in want.items():
        assert tensors[name].shape == a.shape
        assert np.array_equal(np.asarray(tensors[name]), np.asarray(a, np.uint16)), name
        sp = spans[name]
        assert sp.nbytes == a.size * 2
        assert raw[sp.offset:sp.offset + sp.nbytes] == np.asarray(a, np.uint16).tobytes(), name


def _rewrite(src: Path, dst: Path, edit_header=None, gen=None):
    """Copy a checkpoint, optionally editing the safetensors header and generation_config.json."""
    dst.mkdir()
    raw = (src / "model.safetensors").read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    if edit_header:
        header, data = edit_header(header, data)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    (dst / "model.safetensors").write_bytes(struct.pack("<Q", len(hb)) + hb + data)
    (dst / "config.json").write_text((src / "config.json").read_text())
    g = json.loads((src / "generation_config.json").read_text()) if gen is None else gen
    (dst / "generation_config.json").write_text(json.dumps(g))
    return dst


@pytest.mark.parametrize("case", ["missing", "dtype", "shape", "misaligned", "unused", "no_eos", "negative_offset",
                                  "float_offset"])
def test_malformed_checkpoints_are_rejected(tiny, tmp_path, case):
    def edit(header, data):
        name = next(k for k in sorted(header) if k.endswith("q_proj.weight"))
        if case == "missing":
            del header[name]
        elif case == "dtype":
            header[name]["dtype"] = "F16"
        elif case == "shape":
            r, c = header[name]["shape"]
            header[name]["shape"] = [r // 2, c * 2]  # same number of elements, not config.json's shape
        elif case == "misaligned":
            b, e = header[name]["data_offsets"]
            header[name]["data_offsets"] = [b + 2, e + 2]
            data = data + b"\0\0"
        elif case == "negative_offset":  # 16-byte aligned, right length, but before the data
            b, e = header[name]["data_offsets"]
            n = e - b
            header[name]["data_offsets"] = [-16, n - 16]
        elif case == "float_offset":
            b, e = header[name]["data_offsets"]
            header[name]["data_offsets"] = [float(b), float(e)]
        elif case == "unused":
            header["extra.weight"] = {"dtype": "BF16", "shape": [8], "data_offsets": [len(data), len(data) + 16]}
            data = data + bytes(16)
        return header, data

    d = _rewrite(tiny, tmp_path / "bad", edit_header=None if case == "no_eos" else edit,
                 gen={} if case == "no_eos" else None)
    with pytest.raises(ckpt.CheckpointError):
        ckpt.checkpoint_layout(d)


def test_tensor_in_two_shards_is_rejected(tiny, tmp_path):
    """Split the checkpoint into two shards that both hold one tensor."""
    raw = (tiny / "model.safetensors").read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    names = sorted(k for k in header if k != "__metadata__")
    dup = names[0]

    def shard(keys):
        h, blob = {}, b""
        for k in keys:
            b, e = header[k]["data_offsets"]
            pad = (-len(blob)) % 16
            blob += bytes(pad)
            h[k] = dict(header[k], data_offsets=[len(blob), len(blob) + e - b])
            blob += data[b:e]
        hb = json.dumps(h).encode()
        hb += b" " * ((8 - len(hb) % 8) % 8)
        return struct.pack("<Q", len(hb)) + hb + blob

    d = tmp_path / "two"
    d.mkdir()
    half = len(names) // 2
    (d / "model-00001-of-00002.safetensors").write_bytes(shard(names[:half]))
    (d / "model-00002-of-00002.safetensors").write_bytes(shard(names[half:] + [dup]))
    for f in ("config.json", "generation_config.json"):
        (d / f).write_text((tiny / f).read_text())
    with pytest.raises(ckpt.CheckpointError, match="appears in both"):
        ckpt.checkpoint_layout(d)
    # the same two shards without the duplicate load
    (d / "model-00002-of-00002.safetensors").write_bytes(shard(names[half:]))
    shape, spans = ckpt.checkpoint_layout(d)
    assert set(spans) == set(names)


@pytest.mark.gpu
def test_fast_loader_matches_plain_loader(tiny):
    torch = pytest.importorskip("torch")
    from llm_inference_b200.engine import DeviceWeights
    plain = DeviceWeights.from_checkpoint(tiny)
    # one chunk per tensor, and chunks that split tensors; one host thread, and several that
    # share out the chunks
    for staging, threads in ((64 << 20, None), (4096, 1), (4096, 3), (16000, 8)):
        fast = DeviceWeights.load(tiny, staging_bytes=staging, threads=threads)
        assert fast.offsets == plain.offsets
        assert torch.equal(fast.blob, plain.blob), f"staging {staging}, threads {threads}"
