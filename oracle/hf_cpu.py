"""The reference's CPU decode path, timed on the host -- TEST/BASELINE INFRASTRUCTURE ONLY.

The reference's CPU implementation of this path is its Hugging Face transformers harness:
bench/hf_baseline.py:10-24 (``decode``) runs the prompt, then one-token forwards with the KV
cache, taking the argmax and reading it back (``.item()``) every step. This module restates
that loop with the model kept on the CPU (the harness hard-codes .cuda() and
torch.cuda.synchronize(), bench/hf_baseline.py:16,23,37-38), bf16 weights, sdpa attention and
all host threads. It builds a random-init Qwen3 of the requested shape and a KV cache pre-filled
with N(0, 1) values, so one decode step costs what the GPU workload's step costs per sequence.

Only bench.py's cpu_baseline leg and its ``--impl reference`` arm use it, as a reported
baseline; nothing on the product path imports it.
"""
from __future__ import annotations

import os
import time


def _fill(params, seed, std):
    """Fill tensors with N(0, std) values quickly: one random block, tiled."""
    import torch
    g = torch.Generator().manual_seed(seed)
    block = (torch.randn(1 << 22, generator=g) * std).to(torch.bfloat16)
    for p in params:
        flat = p.data.view(-1)
        n = flat.numel()
        for o in range(0, n, block.numel()):
            k = min(block.numel(), n - o)
            flat[o:o + k].copy_(block[:k])


def build(shape, threads: int | None = None, seed: int = 0):
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.set_num_threads(threads or os.cpu_count() or 1)
    cfg = Qwen3Config(hidden_size=shape.hidden_size, intermediate_size=shape.intermediate_size,
                      num_hidden_layers=shape.num_hidden_layers, num_attention_heads=shape.num_attention_heads,
                      num_key_value_heads=shape.num_key_value_heads, head_dim=shape.head_dim,
                      vocab_size=shape.vocab_size, max_position_embeddings=max(shape.max_position_embeddings, 8192),
                      rms_norm_eps=shape.rms_norm_eps, tie_word_embeddings=shape.tie_word_embeddings,
                      rope_parameters={"rope_type": "default", "rope_theta": shape.rope_theta})
    cfg._attn_implementation = "sdpa"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
    model = model.to_empty(device="cpu").to(torch.bfloat16).eval()
    norms = [p for n, p in model.named_parameters() if n.endswith("norm.weight")]
    others = [p for n, p in model.named_parameters() if not n.endswith("norm.weight")]
    _fill(others, seed, 0.02)
    for p in norms:
        p.data.fill_(1.0)
    model.model.rotary_emb.__init__(cfg)  # buffers were created on meta
    return model


def prefilled_cache(model, batch: int, kv_len: int, seed: int = 1):
    """A DynamicCache holding kv_len positions of N(0, 1) keys and values per layer."""
    import torch
    from transformers import DynamicCache

    cfg = model.config
    cache = DynamicCache(config=cfg)
    shape = (batch, cfg.num_key_value_heads, kv_len, cfg.head_dim)
    for layer in range(cfg.num_hidden_layers):
        k = torch.empty(shape, dtype=torch.bfloat16)
        v = torch.empty(shape, dtype=torch.bfloat16)
        _fill([k, v], seed + layer, 1.0)
        cache.update(k, v, layer)
    return cache


def decode_steps(model, cache, tokens, n_steps: int) -> list[float]:
    """bench/hf_baseline.py:18-22 on the CPU: per step one forward of the batch's last tokens with
    the cache, argmax, and a host read of the tokens. Returns the seconds of each step."""
    import torch

    token = torch.tensor(tokens, dtype=torch.long).view(-1, 1)
    times = []
    with torch.inference_mode():
        for _ in range(n_steps):
            t0 = time.perf_counter()
            out = model(input_ids=token, past_key_values=cache, use_cache=True)
            cache = out.past_key_values
            token = out.logits[:, -1].argmax(dim=-1, keepdim=True)
            token.tolist()
            times.append(time.perf_counter() - t0)
    return times
