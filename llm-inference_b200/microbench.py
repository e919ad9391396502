"""Each decode kernel timed alone on one B200 (the isolated fused-kernel microbenchmark).

Default workload: BASELINE configuration 1.
- Qwen3-1.7B shapes (hidden 2048, 16 q / 8 kv heads, head_dim 128, intermediate 6144).
- bf16 N(0, 1) activations at batch 1, 16, 64 and 256.
- Positions uniform in [0, 4096), seeded.

The kernels are rmsnorm, qk_norm_rope with the KV write, gate_up (SwiGLU), gemv_residual
(o_proj and down) and the embedding gather. The projections, LM head, attention and argmax of
the same step can be added with --kernels.

Every launch goes through the C ABI (include/qwen3_b200.h):
- batch 1 uses the drop-in launchers (the reference's parameters);
- batch > 1 uses the batched ones.

Each launch is timed alone with CUDA events on its stream. Before it, a 512 MB buffer is read,
which evicts the 126 MB L2. The line reports the mean over --iters launches, and the
kernel's algorithmic bytes (every byte it must move once) ÷ that time against the measured
copy peak in MEASURED_PEAKS.json.

    python llm-inference_b200/microbench.py [--model qwen3-1.7b] [--batch 1 16 64 256]
        [--kernels rmsnorm qk_norm_rope gate_up o_proj down embedding qkv lm_head attention
                   rope_attention argmax]
        [--kv 4096] [--iters 20] [--warmup 3]

One JSON line per (kernel, batch).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent

DEFAULT_KERNELS = ["rmsnorm", "qk_norm_rope", "gate_up", "o_proj", "down", "embedding"]
ALL_KERNELS = DEFAULT_KERNELS + ["qkv", "lm_head", "attention", "rope_attention", "argmax"]


def _package():
    name = "llm_inference_b200"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, HERE / "__init__.py", submodule_search_locations=[str(HERE)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def hbm_peak() -> tuple[float, str]:
    try:
        return float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


class Bench:
    def __init__(self, args):
        import torch
        self.torch = torch
        _package()
        from llm_inference_b200 import _lib, checkpoint
        self.lib = _lib
        self.s = checkpoint.PRESETS[args.model]
        self.args = args
        self.stream = torch.cuda.Stream()
        self.g = torch.Generator(device="cuda").manual_seed(args.seed)
        self.flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")

    def rn(self, *shape, std=1.0, mean=0.0):
        t = self.torch
        return (t.randn(*shape, generator=self.g, device="cuda") * std + mean).bfloat16()

    def positions(self, batch, kv):
        t = self.torch
        return t.randint(0, kv, (batch,), generator=self.g, device="cuda", dtype=t.int32)

    def time(self, launch) -> float:
        """Mean µs of one launch, each after an L2-evicting read, timed on the bench stream."""
        t = self.torch
        ev = [(t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)) for _ in range(self.args.iters)]
        s = self.stream.cuda_stream
        t.cuda.synchronize()  # the inputs were made on torch's stream, which this one does not follow
        with t.cuda.stream(self.stream):
            for _ in range(self.args.warmup):
                launch(s)
            for e0, e1 in ev:
                self.flush.sum(dtype=t.int64)
                e0.record(self.stream)
                launch(s)
                e1.record(self.stream)
        t.cuda.synchronize()
        return sum(e0.elapsed_time(e1) for e0, e1 in ev) / len(ev) * 1e3

    # --------------------------------------------------------------- kernels: (launch, bytes)
    def k_rmsnorm(self, B):
        H = self.s.hidden_size
        x, w, y = self.rn(B, H), self.rn(H, std=0.02, mean=1.0), self.torch.empty(B, H, dtype=self.torch.bfloat16, device="cuda")
        return (lambda s: self.lib.call("q3_rmsnorm_forward", y.data_ptr(), x.data_ptr(), w.data_ptr(), B, H, 1e-6, s),
                2 * B * H * 2 + H * 2)

    def k_qk_norm_rope(self, B):
        s_ = self.s
        nq, nkv, hd, kv = s_.num_attention_heads, s_.num_key_value_heads, s_.head_dim, self.args.kv
        q, k, v = self.rn(B, nq * hd), self.rn(B, nkv * hd), self.rn(B, nkv * hd)
        qn, kn = self.rn(hd, std=0.02, mean=1.0), self.rn(hd, std=0.02, mean=1.0)
        kc = self.torch.empty(B, kv, nkv * hd, dtype=self.torch.bfloat16, device="cuda")
        vc = self.torch.empty_like(kc)
        pos = self.positions(B, kv)
        strides = (kv * nkv * hd, nkv * hd, hd)  # the reference's cache layout
        if B == 1:
            def launch(s):
                self.lib.call("q3_qk_norm_rope_forward", q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr(),
                              kn.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), nq, nkv, hd, 1e-6,
                              s_.rope_theta, None, None, s)
        else:
            def launch(s):
                self.lib.call("q3_qk_norm_rope_batched", q.data_ptr(), k.data_ptr(), v.data_ptr(), qn.data_ptr(),
                              kn.data_ptr(), kc.data_ptr(), vc.data_ptr(), *strides, pos.data_ptr(), B, nq, nkv, hd,
                              kv, 1e-6, s_.rope_theta, None, None, s)
        per_seq = 2 * nq * hd * 2 + 2 * nkv * hd * 2 + nkv * hd * 2 + 2 * nkv * hd * 2
        return launch, B * per_seq + 2 * hd * 2

    def _proj(self, B, rows, cols, kind):
        t = self.torch
        x = self.rn(B, cols)
        if kind == "gate_up":
            wg, wu = self.rn(rows, cols, std=0.02), self.rn(rows, cols, std=0.02)
            act = t.empty(B, rows, dtype=t.bfloat16, device="cuda")
            if B == 1:
                f = lambda s: self.lib.call("q3_gate_up_forward", act.data_ptr(), wg.data_ptr(), wu.data_ptr(),
                                            x.data_ptr(), rows, cols, None, None, s)
            else:
                f = lambda s: self.lib.call("q3_gate_up_batched", act.data_ptr(), wg.data_ptr(), wu.data_ptr(),
                                            x.data_ptr(), B, rows, cols, None, None, s)
            return f, 2 * rows * cols * 2 + B * cols * 2 + B * rows * 2
        w = self.rn(rows, cols, std=0.02)
        if kind == "residual":
            res = self.rn(B, rows)
            if B == 1:
                f = lambda s: self.lib.call("q3_gemv_residual_forward", res.data_ptr(), w.data_ptr(), x.data_ptr(),
                                            rows, cols, None, s)
            else:
                f = lambda s: self.lib.call("q3_gemv_residual_batched", res.data_ptr(), w.data_ptr(), x.data_ptr(),
                                            B, rows, cols, None, s)
            return f, rows * cols * 2 + B * cols * 2 + 2 * B * rows * 2
        out = t.empty(B, rows, dtype=t.bfloat16, device="cuda")
        if B == 1:
            f = lambda s: self.lib.call("q3_gemv_forward", out.data_ptr(), w.data_ptr(), x.data_ptr(), rows, cols, s)
        else:
            f = lambda s: self.lib.call("q3_gemv_batched", out.data_ptr(), w.data_ptr(), x.data_ptr(), B, rows, cols, s)
        return f, rows * cols * 2 + B * cols * 2 + B * rows * 2

    def k_gate_up(self, B):
        return self._proj(B, self.s.intermediate_size, self.s.hidden_size, "gate_up")

    def k_o_proj(self, B):
        return self._proj(B, self.s.hidden_size, self.s.num_attention_heads * self.s.head_dim, "residual")

    def k_down(self, B):
        return self._proj(B, self.s.hidden_size, self.s.intermediate_size, "residual")

    def k_lm_head(self, B):
        return self._proj(B, self.s.vocab_size, self.s.hidden_size, "plain")

    def k_qkv(self, B):
        t, s_ = self.torch, self.s
        H, Q, KV = s_.hidden_size, s_.num_attention_heads * s_.head_dim, s_.num_key_value_heads * s_.head_dim
        x = self.rn(B, H)
        wq, wk, wv = self.rn(Q, H, std=0.02), self.rn(KV, H, std=0.02), self.rn(KV, H, std=0.02)
        q, k, v = (t.empty(B, n, dtype=t.bfloat16, device="cuda") for n in (Q, KV, KV))
        if B == 1:
            f = lambda s: self.lib.call("q3_qkv_forward", q.data_ptr(), k.data_ptr(), v.data_ptr(), wq.data_ptr(),
                                        wk.data_ptr(), wv.data_ptr(), x.data_ptr(), Q, KV, H, s)
        else:
            f = lambda s: self.lib.call("q3_qkv_batched", q.data_ptr(), k.data_ptr(), v.data_ptr(), wq.data_ptr(),
                                        wk.data_ptr(), wv.data_ptr(), x.data_ptr(), B, Q, KV, H, s)
        return f, (Q + 2 * KV) * H * 2 + B * H * 2 + B * (Q + 2 * KV) * 2

    def k_embedding(self, B):
        t, s_ = self.torch, self.s
        V, H = s_.vocab_size, s_.hidden_size
        table = self.rn(V, H, std=0.02)
        toks = t.randint(0, V, (B,), generator=self.g, device="cuda", dtype=t.int32)
        out = t.empty(B, H, dtype=t.bfloat16, device="cuda")
        if B == 1:
            f = lambda s: self.lib.call("q3_embedding_forward", out.data_ptr(), table.data_ptr(), toks.data_ptr(), H, s)
        else:
            f = lambda s: self.lib.call("q3_embedding_batched", out.data_ptr(), table.data_ptr(), toks.data_ptr(), B,
                                        H, V, s)
        return f, 2 * B * H * 2

    def k_argmax(self, B):
        t, V = self.torch, self.s.vocab_size
        x = self.rn(B, V)
        out = t.empty(B, dtype=t.int32, device="cuda")
        if B == 1:
            f = lambda s: self.lib.call("q3_argmax_forward", out.data_ptr(), x.data_ptr(), V, s)
        else:
            f = lambda s: self.lib.call("q3_argmax_batched", out.data_ptr(), x.data_ptr(), B, V, s)
        return f, B * V * 2

    def k_attention(self, B):
        """Batched split attention over head-major caches; every sequence at position --kv - 1
        (the bench workload's shape when --kv 4096 --batch 32 --model qwen3-4b)."""
        t, s_ = self.torch, self.s
        nq, nkv, hd, L = s_.num_attention_heads, s_.num_key_value_heads, s_.head_dim, self.args.kv
        max_seq = L
        kc = self.rn(B, nkv, max_seq, hd)
        vc = self.rn(B, nkv, max_seq, hd)
        q = self.rn(B, nq * hd)
        out = t.empty_like(q)
        pos = t.full((B,), L - 1, dtype=t.int32, device="cuda")
        nbytes = self.lib.load().q3_attention_scratch_bytes(B, nq, nkv, hd, max_seq)
        scratch = t.empty(nbytes, dtype=t.uint8, device="cuda")
        strides = (nkv * max_seq * hd, hd, max_seq * hd)
        scale = 1.0 / math.sqrt(hd)
        f = lambda s: self.lib.call("q3_attention_batched", out.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                    *strides, scratch.data_ptr(), pos.data_ptr(), B, nq, nkv, hd, max_seq, scale, s)
        return f, B * L * nkv * hd * 2 * 2 + 2 * B * nq * hd * 2

    def k_rope_attention(self, B):
        """RoPE + attention in one launch (q3_rope_attention_batched, the engine's path for small
        batches) over head-major caches; every sequence at position --kv - 1. None when the fused
        kernel does not apply to the batch."""
        t, s_ = self.torch, self.s
        nq, nkv, hd, L = s_.num_attention_heads, s_.num_key_value_heads, s_.head_dim, self.args.kv
        max_seq = L
        chunks = self.lib.load().q3_rope_attention_chunks(B, nq, nkv, hd, max_seq)
        if chunks <= 0:
            return None
        kc = self.rn(B, nkv, max_seq, hd)
        vc = self.rn(B, nkv, max_seq, hd)
        q, k, v = self.rn(B, nq * hd), self.rn(B, nkv * hd), self.rn(B, nkv * hd)
        qn, kn = self.rn(hd, std=0.02, mean=1.0), self.rn(hd, std=0.02, mean=1.0)
        out = t.empty_like(q)
        pos = t.full((B,), L - 1, dtype=t.int32, device="cuda")
        strides = (nkv * max_seq * hd, hd, max_seq * hd)
        scale = 1.0 / math.sqrt(hd)
        f = lambda s: self.lib.call("q3_rope_attention_batched", out.data_ptr(), q.data_ptr(), k.data_ptr(),
                                    v.data_ptr(), qn.data_ptr(), kn.data_ptr(), kc.data_ptr(), vc.data_ptr(), *strides,
                                    pos.data_ptr(), B, nq, nkv, hd, max_seq, 1e-6, s_.rope_theta, scale, chunks, s)
        self.extra = {"chunks": chunks}
        # K and V rows of positions 0..L-2 read, q/k/v read, the output and two cache rows written
        return f, B * (L - 1) * nkv * hd * 2 * 2 + B * (2 * nq + 4 * nkv) * hd * 2


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--model", default="qwen3-1.7b")
    ap.add_argument("--batch", type=int, nargs="+", default=[1, 16, 64, 256])
    ap.add_argument("--kernels", nargs="+", default=DEFAULT_KERNELS, choices=ALL_KERNELS)
    ap.add_argument("--kv", type=int, default=4096, help="positions: uniform in [0, kv) (attention: all at kv-1)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    if args.warmup < 1 or args.iters < 1:
        ap.error("--warmup and --iters must be positive")
    b = Bench(args)
    peak, source = hbm_peak()
    q3 = sys.modules["llm_inference_b200"]
    for name in args.kernels:
        for B in args.batch:
            b.extra = {}
            made = getattr(b, "k_" + name)(B)
            if made is None:
                print(json.dumps({"kernel": name, "model": args.model, "batch": B, "skipped": "not applicable"}),
                      flush=True)
                continue
            launch, nbytes = made
            us = b.time(launch)
            gbs = nbytes / (us * 1e-6) / 1e9
            if q3.device_error() != 0:
                raise SystemExit(f"{name} batch {B}: device error flags set")
            print(json.dumps({"kernel": name, "model": args.model, "batch": B, "us": round(us, 2),
                              "algorithmic_bytes": int(nbytes), "gbs": round(gbs, 1), "peak_gbs": peak,
                              "frac": round(gbs / peak, 4), "peak_source": source, **b.extra}), flush=True)
            b.torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
