"""Qwen3 checkpoints in the reference engine's on-disk layout.

The reference engine reads a model directory holding ``config.json``,
``generation_config.json`` and one or more ``*.safetensors`` shards
(src/loader.cu:105-139, :73-103, :141-216). This module

* writes random-init checkpoints in that layout (:func:`write_random_checkpoint`): seed 0
  by default, linear weights N(0, 0.02), norm weights 1 + N(0, 0.02), drawn with a CPU
  ``torch.Generator`` in sorted tensor-name order and stored as bf16. ``config.json``
  carries a top-level ``rope_theta`` because the reference loader reads that key
  (src/loader.cu:123);
* reads such a directory back (:func:`read_checkpoint`) with the checks the reference
  loader makes (src/loader.cu:239-289, :364-372): BF16 dtype, shapes implied by
  ``config.json``, 16-byte aligned data offsets, and no unused tensors.

Shapes come from the presets in :data:`PRESETS`, named after the models of the
benchmark configurations.
"""
from __future__ import annotations

import json
import struct
from dataclasses import asdict, dataclass, field
from pathlib import Path

import numpy as np


@dataclass
class Qwen3Shape:
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    vocab_size: int
    max_position_embeddings: int = 40960
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    tie_word_embeddings: bool = True
    eos_token_id: list = field(default_factory=lambda: [151645, 151643])

    @property
    def q_dim(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.num_key_value_heads * self.head_dim


PRESETS = {
    "qwen3-0.6b": Qwen3Shape(1024, 3072, 28, 16, 8, 128, 151936),
    "qwen3-1.7b": Qwen3Shape(2048, 6144, 28, 16, 8, 128, 151936),
    "qwen3-4b": Qwen3Shape(2560, 9728, 36, 32, 8, 128, 151936),
    # small shapes for tests: the same structure with GQA, any head_dim the kernels accept
    "tiny": Qwen3Shape(256, 768, 2, 4, 2, 64, 1024, max_position_embeddings=2048,
                       eos_token_id=[1023]),
}


def tensor_shapes(s: Qwen3Shape) -> dict[str, tuple[int, ...]]:
    """Every tensor of a Qwen3 checkpoint with its shape (src/loader.cu:336-362)."""
    shapes = {"model.embed_tokens.weight": (s.vocab_size, s.hidden_size),
              "model.norm.weight": (s.hidden_size,)}
    for l in range(s.num_hidden_layers):
        p = f"model.layers.{l}."
        shapes[p + "input_layernorm.weight"] = (s.hidden_size,)
        shapes[p + "self_attn.q_proj.weight"] = (s.q_dim, s.hidden_size)
        shapes[p + "self_attn.k_proj.weight"] = (s.kv_dim, s.hidden_size)
        shapes[p + "self_attn.v_proj.weight"] = (s.kv_dim, s.hidden_size)
        shapes[p + "self_attn.q_norm.weight"] = (s.head_dim,)
        shapes[p + "self_attn.k_norm.weight"] = (s.head_dim,)
        shapes[p + "self_attn.o_proj.weight"] = (s.hidden_size, s.q_dim)
        shapes[p + "post_attention_layernorm.weight"] = (s.hidden_size,)
        shapes[p + "mlp.gate_proj.weight"] = (s.intermediate_size, s.hidden_size)
        shapes[p + "mlp.up_proj.weight"] = (s.intermediate_size, s.hidden_size)
        shapes[p + "mlp.down_proj.weight"] = (s.hidden_size, s.intermediate_size)
    if not s.tie_word_embeddings:
        shapes["lm_head.weight"] = (s.vocab_size, s.hidden_size)
    return shapes


def is_norm(name: str) -> bool:
    return name.endswith("norm.weight")


def random_tensors(s: Qwen3Shape, seed: int = 0) -> dict[str, np.ndarray]:
    """Random-init weights as bf16 bit arrays (uint16), in sorted-name draw order."""
    import torch

    g = torch.Generator().manual_seed(seed)
    out = {}
    for name in sorted(tensor_shapes(s)):
        shape = tensor_shapes(s)[name]
        t = torch.randn(shape, generator=g, dtype=torch.float32) * 0.02
        if is_norm(name):
            t = t + 1.0
        out[name] = t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return out


def config_json(s: Qwen3Shape) -> dict:
    d = asdict(s)
    eos = d.pop("eos_token_id")
    d.update({
        "architectures": ["Qwen3ForCausalLM"],
        "model_type": "qwen3",
        "hidden_act": "silu",
        "attention_bias": False,
        "attention_dropout": 0.0,
        "torch_dtype": "bfloat16",
        "bos_token_id": eos[-1],
        "eos_token_id": eos[-1],
        # transformers 5 reads rope_parameters, the reference loader the top-level key
        "rope_parameters": {"rope_type": "default", "rope_theta": s.rope_theta},
        "use_cache": True,
        "use_sliding_window": False,
    })
    return d


def write_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    header = {}
    offset = 0
    names = sorted(tensors)
    for name in names:
        a = tensors[name]
        nbytes = a.size * 2
        # the reference loader requires 16-byte aligned offsets (src/loader.cu:273-275)
        assert offset % 16 == 0 and nbytes % 16 == 0, name
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * (-(len(blob) + 8) % 16)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for name in names:
            f.write(np.ascontiguousarray(tensors[name], dtype=np.uint16).tobytes())


def write_random_checkpoint(out_dir, shape: Qwen3Shape | str, seed: int = 0) -> Path:
    """Write a random-init checkpoint directory readable by the reference engine."""
    s = PRESETS[shape] if isinstance(shape, str) else shape
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    write_safetensors(out / "model.safetensors", random_tensors(s, seed))
    (out / "config.json").write_text(json.dumps(config_json(s), indent=1))
    (out / "generation_config.json").write_text(json.dumps({"eos_token_id": s.eos_token_id}))
    return out


class CheckpointError(ValueError):
    pass


def shape_from_config(cfg: dict) -> Qwen3Shape:
    """src/loader.cu:105-139: the keys the reference reads, with its checks."""
    try:
        s = Qwen3Shape(
            hidden_size=int(cfg["hidden_size"]), intermediate_size=int(cfg["intermediate_size"]),
            num_hidden_layers=int(cfg["num_hidden_layers"]),
            num_attention_heads=int(cfg["num_attention_heads"]),
            num_key_value_heads=int(cfg["num_key_value_heads"]), head_dim=int(cfg["head_dim"]),
            vocab_size=int(cfg["vocab_size"]),
            max_position_embeddings=int(cfg["max_position_embeddings"]),
            rms_norm_eps=float(cfg["rms_norm_eps"]), rope_theta=float(cfg["rope_theta"]),
            tie_word_embeddings=cfg["tie_word_embeddings"])
    except KeyError as e:
        raise CheckpointError(f'config.json has no number "{e.args[0]}"') from None
    if not isinstance(s.tie_word_embeddings, bool):
        raise CheckpointError('config.json has no bool "tie_word_embeddings"')
    if s.num_attention_heads % s.num_key_value_heads != 0:
        raise CheckpointError("num_attention_heads must be a multiple of num_key_value_heads")
    return s


@dataclass
class TensorSpan:
    """Where one tensor's bytes lie: `nbytes` bytes at byte `offset` of file `path`."""
    path: Path
    offset: int
    nbytes: int
    shape: tuple[int, ...]


def checkpoint_layout(model_dir) -> tuple[Qwen3Shape, dict[str, TensorSpan]]:
    """Validate a checkpoint directory from its config files and safetensors headers alone (the
    tensor data is not read) and locate every tensor the engine uses. The checks are those of
    src/loader.cu:113-140 and :313-380: config fields, an eos token, BF16 dtype, shapes implied
    by config.json, data offsets inside the file, 16-byte alignment, no unused tensors (a tied
    checkpoint may carry lm_head.weight)."""
    d = Path(model_dir)
    s = shape_from_config(json.loads((d / "config.json").read_text()))
    gen = json.loads((d / "generation_config.json").read_text())
    eos = gen.get("eos_token_id")
    s.eos_token_id = [eos] if isinstance(eos, int) else list(eos or [])
    if not s.eos_token_id:
        raise CheckpointError("generation_config.json has no \"eos_token_id\"")
    files = sorted(d.glob("*.safetensors"))
    if not files:
        raise CheckpointError(f"no .safetensors files in {d}")
    entries = {}
    for p in files:
        size = p.stat().st_size
        with open(p, "rb") as f:
            head = f.read(8)
            if len(head) < 8:
                raise CheckpointError(f"{p}: too small to be a safetensors file")
            (n,) = struct.unpack("<Q", head)
            if n > size - 8:
                raise CheckpointError(f"{p}: bad header length")
            header = json.loads(f.read(n))
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            if name in entries:  # the reference's lookup would take the first file's copy
                raise CheckpointError(f"tensor {name} appears in both {entries[name][1].name} and {p.name}")
            entries[name] = (meta, p, 8 + n, size - 8 - n)
    want = tensor_shapes(s)
    spans = {}
    for name, shape in want.items():
        if name not in entries:
            raise CheckpointError(f"tensor {name} not found")
        meta, path, data_start, data_len = entries[name]
        if meta.get("dtype") != "BF16":
            raise CheckpointError(f"{name}: dtype is not BF16")
        if tuple(meta["shape"]) != shape:
            raise CheckpointError(f"{name}: shape {meta['shape']}, config.json implies {list(shape)}")
        offs = meta.get("data_offsets")
        if (not isinstance(offs, list) or len(offs) != 2
                or not all(isinstance(o, int) and not isinstance(o, bool) for o in offs)):
            raise CheckpointError(f"{name}: data_offsets must be two integers")
        b, e = offs
        if b < 0 or e > data_len or e - b != int(np.prod(shape)) * 2:
            raise CheckpointError(f"{name}: data_offsets do not match its shape")
        if b % 16:
            raise CheckpointError(f"{name}: offset {b} is not 16-byte aligned")
        spans[name] = TensorSpan(path, data_start + b, e - b, shape)
    allowed = 1 if (s.tie_word_embeddings and "lm_head.weight" in entries) else 0
    unused = len(entries) - len(spans)
    if unused != allowed:
        raise CheckpointError(f"{unused} tensors in the safetensors files are not used by the engine")
    return s, spans


def read_checkpoint(model_dir) -> tuple[Qwen3Shape, dict[str, np.ndarray]]:
    """Read and validate a checkpoint directory; tensors are bf16 bit arrays (views of the
    memory-mapped files)."""
    s, spans = checkpoint_layout(model_dir)
    maps = {}
    tensors = {}
    for name, sp in spans.items():
        if sp.path not in maps:
            maps[sp.path] = np.memmap(sp.path, dtype=np.uint8, mode="r")
        tensors[name] = maps[sp.path][sp.offset:sp.offset + sp.nbytes].view(np.uint16).reshape(sp.shape)
    return s, tensors


def weight_checksums(tensors: dict[str, np.ndarray]) -> dict[str, tuple[int, int, int]]:
    """Per tensor: (numel, sum of bf16 bits, position-weighted sum) mod 2^64, as
    print_weight_checksums (src/loader.cu:395-419) and ref/weight_checksums.py compute."""
    out = {}
    with np.errstate(over="ignore"):
        for name, a in tensors.items():
            bits = np.ascontiguousarray(a).reshape(-1).astype(np.uint64)
            idx = np.arange(1, bits.size + 1, dtype=np.uint64)
            out[name] = (bits.size, int(bits.sum(dtype=np.uint64)), int((idx * bits).sum(dtype=np.uint64)))
    return out
