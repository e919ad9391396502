"""The reference's batch-1 forward pass, composed from its own CUDA kernels -- TEST INFRASTRUCTURE ONLY.

``RefForward`` runs src/forward.cu:118-193 (``forward_kernels``) launch for launch on the GPU
through ``oracle/_ref/libqwen3_ref.so`` (the reference's src/kernels.cu compiled for sm_100a,
see ``ref_kernels.py``): embedding, then per layer rmsnorm, qkv, qk_norm_rope (K/V into the
cache slot of the position), attention, gemv_residual (o_proj), rmsnorm, gate_up,
gemv_residual (down), then the final rmsnorm, the LM-head gemv and argmax
(src/forward.cu:229-236). One instance is one sequence with its own caches in the reference's
layout, ``[n_layers][max_seq][n_kv*head_dim]`` (src/forward.cuh:15-16), so any max_seq works
(the reference engine caps it at 4096 in src/forward.cu:8; its kernels do not).

It reads the weights where a :class:`DeviceWeights` keeps them, so the engine under test and this
oracle see the same bytes. The GPU parity tests use it at the benchmark's shapes, where the CPU
oracle (qwen3_oracle.c) would take minutes per token.
"""
from __future__ import annotations

import math

import numpy as np

import ref_kernels


class RefForward:
    def __init__(self, weights, max_seq: int):
        import torch
        self.w = weights
        s = weights.shape
        self.s = s
        self.max_seq = max_seq
        self.q_dim = s.num_attention_heads * s.head_dim
        self.kv_dim = s.num_key_value_heads * s.head_dim
        dev = "cuda"
        bf = torch.bfloat16
        self.x = torch.empty(s.hidden_size, dtype=bf, device=dev)
        self.xb = torch.empty_like(self.x)
        self.q = torch.empty(self.q_dim, dtype=bf, device=dev)
        self.k = torch.empty(self.kv_dim, dtype=bf, device=dev)
        self.v = torch.empty(self.kv_dim, dtype=bf, device=dev)
        self.attn_out = torch.empty(self.q_dim, dtype=bf, device=dev)
        self.hb = torch.empty(s.intermediate_size, dtype=bf, device=dev)
        self.logits = torch.empty(s.vocab_size, dtype=bf, device=dev)
        self.att = torch.empty(s.num_attention_heads * max_seq, dtype=torch.float32, device=dev)
        self.kc = torch.zeros(s.num_hidden_layers, max_seq, self.kv_dim, dtype=bf, device=dev)
        self.vc = torch.zeros_like(self.kc)
        self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.best = torch.zeros(1, dtype=torch.int32, device=dev)
        self.scale = float(np.float32(1.0 / math.sqrt(s.head_dim)))

    def _p(self, l, suffix):
        return self.w.ptr[f"model.layers.{l}.{suffix}"]

    def forward(self, token: int, pos: int, stream: int = 0):
        """Logits of `token` at `pos` (a device tensor, valid after the stream is synchronized)."""
        s, C = self.s, ref_kernels.call
        H, I = s.hidden_size, s.intermediate_size
        eps, theta = float(np.float32(s.rms_norm_eps)), float(np.float32(s.rope_theta))
        self.tok.fill_(int(token))
        self.pos.fill_(int(pos))
        C("embedding_forward", self.x.data_ptr(), self.w.ptr["model.embed_tokens.weight"], self.tok.data_ptr(), H, stream)
        for l in range(s.num_hidden_layers):
            C("rmsnorm_forward", self.xb.data_ptr(), self.x.data_ptr(), self._p(l, "input_layernorm.weight"), 1, H,
              eps, stream)
            C("qkv_forward", self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), self._p(l, "self_attn.q_proj.weight"),
              self._p(l, "self_attn.k_proj.weight"), self._p(l, "self_attn.v_proj.weight"), self.xb.data_ptr(),
              self.q_dim, self.kv_dim, H, stream)
            C("qk_norm_rope_forward", self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(),
              self._p(l, "self_attn.q_norm.weight"), self._p(l, "self_attn.k_norm.weight"), self.kc[l].data_ptr(),
              self.vc[l].data_ptr(), self.pos.data_ptr(), s.num_attention_heads, s.num_key_value_heads, s.head_dim,
              eps, theta, None, None, stream)
            C("attention_forward", self.attn_out.data_ptr(), self.q.data_ptr(), self.kc[l].data_ptr(),
              self.vc[l].data_ptr(), self.att.data_ptr(), s.num_attention_heads, s.num_key_value_heads, s.head_dim,
              self.pos.data_ptr(), self.max_seq, self.scale, stream)
            C("gemv_residual_forward", self.x.data_ptr(), self._p(l, "self_attn.o_proj.weight"),
              self.attn_out.data_ptr(), H, self.q_dim, None, stream)
            C("rmsnorm_forward", self.xb.data_ptr(), self.x.data_ptr(), self._p(l, "post_attention_layernorm.weight"),
              1, H, eps, stream)
            C("gate_up_forward", self.hb.data_ptr(), self._p(l, "mlp.gate_proj.weight"), self._p(l, "mlp.up_proj.weight"),
              self.xb.data_ptr(), I, H, None, None, stream)
            C("gemv_residual_forward", self.x.data_ptr(), self._p(l, "mlp.down_proj.weight"), self.hb.data_ptr(), H, I,
              None, stream)
        C("rmsnorm_forward", self.xb.data_ptr(), self.x.data_ptr(), self.w.ptr["model.norm.weight"], 1, H, eps, stream)
        lm = self.w.ptr["model.embed_tokens.weight"] if s.tie_word_embeddings else self.w.ptr["lm_head.weight"]
        C("gemv_forward", self.logits.data_ptr(), lm, self.xb.data_ptr(), s.vocab_size, H, stream)
        return self.logits

    def argmax(self, stream: int = 0) -> int:
        ref_kernels.call("argmax_forward", self.best.data_ptr(), self.logits.data_ptr(), self.s.vocab_size, stream)
        return int(self.best.item())
