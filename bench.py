"""Decode throughput benchmark (one JSON line on rank 0).

Workload: Qwen3-4B, random-init on the device from seed 0,
32 independent sequences per GPU, every layer's KV cache pre-filled with bf16 N(0, 1) up to
position 4096, greedy decode. One step decodes one token for every sequence of the GPU.
Sequences are sharded data-parallel: each rank holds a full weight replica and its own 32
sequences, with no collective on the decode path (weak scaling).

  value  tokens/s of all ranks with everything resident on the device: the captured decode
         step replayed back to back (argmax feeds the next step on the device).
  e2e    the same through the C ABI's per-token protocol with host buffers, as the reference
         engine runs (src/forward.cu:206-236): every step copies the tokens and positions from
         pinned host memory, runs the step and copies the argmax tokens back, then syncs.

Timing: W warm-up steps, then K timed steps bracketed by a barrier and a device synchronize,
CUDA events on the engine's stream, the maximum over ranks. Inputs (8 GB of weights, 20 GB of
KV per GPU) exceed the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "llm-inference_b200"

MODEL = "qwen3-4b"
BATCH_PER_GPU = 32
KV_PREFILL = 4096
METRIC = "decode tok/s (Qwen3-4B, 32 seq/GPU, KV 4096, greedy)"
ATTN_TRAFFIC_BYTES = 591_933_696  # measured DRAM bytes of one attention launch (ncu)


def _package():
    name = "llm_inference_b200"
    if name not in sys.modules:
        spec = importlib.util.spec_from_file_location(name, PKG_DIR / "__init__.py",
                                                      submodule_search_locations=[str(PKG_DIR)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name] = mod
        spec.loader.exec_module(mod)
    return sys.modules[name]


def workload_config(n_gpus: int) -> dict:
    return {"workload": "BASELINE config 4: Qwen3-4B random-init, 32 sequences per GPU, KV pre-filled "
                        "bf16 N(0,1) to position 4096, greedy decode",
            "model": MODEL, "batch_per_gpu": BATCH_PER_GPU, "global_batch": BATCH_PER_GPU * n_gpus,
            "kv_prefill": KV_PREFILL, "parallelism": f"dp{n_gpus}",
            "l2": "no flush: weights 8.0 GB and KV 19.6 GB per GPU per step exceed the 126 MB L2"}


# ---------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clock and throttle-reason samples every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- distributed plumbing

class Dist:
    """One process per GPU (RANK / LOCAL_RANK / WORLD_SIZE from torch.distributed.run). The process
    group only brackets the timed regions and takes the maximum time over ranks: decode sequences
    are independent, so nothing is exchanged on the decode path. NCCL on GPUs; gloo on a host
    without CUDA (the CPU tests of this plumbing)."""

    def __init__(self, n_gpus: int):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus:
            raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={self.world}: launch N>1 with torch.distributed.run")
        cuda = torch.cuda.is_available()
        if cuda:
            torch.cuda.set_device(self.local_rank)
        self.device = "cuda" if cuda else "cpu"
        self.pg = None
        if self.world > 1:
            import torch.distributed as dist
            if cuda:
                dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                        device_id=torch.device("cuda", self.local_rank))
            else:
                dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if not self.pg:
            return value
        import torch
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()
            self.pg = None


def timed(dist, stream, fn, name: str) -> float:
    """ms of fn() on `stream`, barrier and synchronize on both sides, max over ranks. The launches
    sit in an NVTX range `name`, so a profiler can select the timed region alone
    (ncu --nvtx --nvtx-include "<name>/")."""
    import torch
    s = torch.cuda.ExternalStream(stream)
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push(name)
    e0.record(s)
    fn()
    e1.record(s)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(e0.elapsed_time(e1))


# ---------------------------------------------------------------- CPU baseline

def cpu_baseline(steps: int = 3) -> dict:
    """The reference's CPU path (HF transformers decode loop) on a bounded sample: one sequence of
    the workload (Qwen3-4B, KV 4096), `steps` decode tokens, all host threads."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import hf_cpu
    from llm_inference_b200 import checkpoint
    shape = checkpoint.PRESETS[MODEL]
    cores = os.cpu_count() or 1
    model = hf_cpu.build(shape, threads=cores)
    cache = hf_cpu.prefilled_cache(model, 1, KV_PREFILL)
    times = hf_cpu.decode_steps(model, cache, [17], steps + 1)[1:]  # first step warms up
    sec = statistics.median(times)
    return {"value": round(1.0 / sec, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
            "sample": f"HF transformers Qwen3ForCausalLM bf16 on CPU (decode loop of bench/hf_baseline.py:10-24), "
                      f"1 sequence at KV {KV_PREFILL}, median of {steps} decode steps"}


# ---------------------------------------------------------------- arms

def run_mine(args) -> dict | None:
    import torch
    q3 = _package()
    from llm_inference_b200 import checkpoint
    from llm_inference_b200.engine import DeviceWeights, Engine

    dist = Dist(args.gpus)
    shape = checkpoint.PRESETS[MODEL]
    B, K, W = BATCH_PER_GPU, args.steps, args.warmup
    max_seq = KV_PREFILL + 2 * (W + K) + 16
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        weights = DeviceWeights.random(shape, seed=0)
        eng = Engine(weights, batch=B, max_seq=max_seq, history_cap=2 * (W + K) + 8, stream=stream.cuda_stream)
        eng.fill_kv_normal(KV_PREFILL, seed=1000 + dist.rank)
        import numpy as np
        rng = np.random.default_rng(dist.rank)
        eng.set_state(rng.integers(0, shape.vocab_size, B).tolist(), [KV_PREFILL] * B)
        eng.capture()
        eng.step(W)
    torch.cuda.synchronize()

    with ClockSampler(torch.cuda.current_device()) as clk:
        ms = timed(dist, stream.cuda_stream, lambda: eng.step(K), "decode_steps")
        # e2e: the per-token host protocol, continuing from the device loop's state
        toks = eng.sample_argmax()
        pos0 = KV_PREFILL + W + K
        def e2e():
            t = toks
            for i in range(K):
                eng.forward(t, [pos0 + i] * B)
                t = eng.sample_argmax()
        ms_e2e = timed(dist, stream.cuda_stream, e2e, "decode_e2e")
    clocks = clk.summary()
    if q3.device_error(stream.cuda_stream) != 0:
        raise SystemExit("device error flags set during the benchmark")

    n = dist.world
    tok = n * B * K
    weight_bytes = eng.weight_bytes_per_step()
    kvpp = eng.kv_bytes_per_position()
    mean_ctx = KV_PREFILL + W + (K + 1) / 2  # positions attended per sequence, averaged over the timed steps
    step_bytes = weight_bytes + B * kvpp * mean_ctx
    line = None
    if dist.rank == 0:
        import json as _j
        peaks = {}
        try:
            peaks = _j.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        except (OSError, ValueError):
            pass
        hbm = peaks.get("hbm_gbs", 6650.0)
        step_gbs = step_bytes / (ms / K * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": round(tok / (ms * 1e-3), 1), "unit": "tok/s", "n_gpus": n, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) KV, random ids)",
            "config": workload_config(n),
            "clocks": clocks,
            "e2e": {"value": round(tok / (ms_e2e * 1e-3), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": 2 * B * 4, "d2h_bytes_per_step": B * 4},
            "gpu_launches": eng.launches_per_step() * K,
            "step_roofline": {"bound": "hbm", "bytes_per_step": int(step_bytes), "achieved": round(step_gbs, 1),
                              "peak": hbm, "unit": "GB/s", "frac": round(step_gbs / hbm, 4),
                              "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"},
        }
        line["roofline"] = kernel_roofline(eng, stream, hbm, "hbm_gbs" in peaks)
    eng.close()
    dist.close()
    return line


def kernel_roofline(eng, stream, hbm_peak, measured) -> dict:
    """Dominant kernel (attention over the KV cache: 70 % of a step's bytes) timed alone with CUDA
    events on the engine's stream at the benchmark's state; achieved = algorithmic bytes / time."""
    import torch
    from llm_inference_b200 import _lib
    s = eng.shape
    B = eng.batch
    kvd = s.num_key_value_heads * s.head_dim
    pos = eng.positions().clone()
    ctx = float((pos.double() + 1).mean())
    buf = eng.info
    nbytes = _lib.load().q3_attention_scratch_bytes(B, s.num_attention_heads, s.num_key_value_heads, s.head_dim,
                                                    eng.max_seq)
    scratch = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    q = torch.randn(B, s.num_attention_heads * s.head_dim, device="cuda").bfloat16()
    out = torch.empty_like(q)
    scale = 1.0 / s.head_dim ** 0.5
    layer_stride = B * eng.max_seq * kvd * 2  # bytes between layers' caches
    hd = s.head_dim  # the engine's caches are head-major: [B][n_kv][max_seq][head_dim] per layer
    reps = 20
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ts = torch.cuda.ExternalStream(stream.cuda_stream)
    for i in range(3 + reps):
        if i == 3:
            ev0.record(ts)
        layer = i % s.num_hidden_layers  # a different layer's cache each launch: no L2 reuse
        _lib.call("q3_attention_batched", out.data_ptr(), q.data_ptr(), buf.key_cache + layer * layer_stride,
                  buf.value_cache + layer * layer_stride, eng.max_seq * kvd, hd, eng.max_seq * hd,
                  scratch.data_ptr(), pos.data_ptr(), B,
                  s.num_attention_heads, s.num_key_value_heads, s.head_dim, eng.max_seq, scale, stream.cuda_stream)
    ev1.record(ts)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / reps
    alg = B * ctx * kvd * 2 * 2  # K and V rows read once per launch
    gbs = alg / (ms * 1e-3) / 1e9
    return {"kernel": "attention (q3_attention_batched: scores + pv kernels), one layer, 32 sequences",
            "bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
            "algorithmic_bytes_per_launch": int(alg), "us_per_launch": round(ms * 1e3, 2),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if measured else "fallback",
            # dram__bytes_read.sum + dram__bytes_write.sum of the four attention kernels of one
            # launch at this exact shape, from an ncu capture
            "traffic": ATTN_TRAFFIC_BYTES, "traffic_source": "ncu capture, one launch at position 4095"}


def run_config3(args) -> dict | None:
    """Qwen3-4B at batch 1, greedy decode, tok/s at positions 256, 2048
    and 8192 (the cache before each position pre-filled with bf16 N(0, 1), standing in for the
    tokens a real decode would have written). One engine, one captured step, replayed K times at
    each position; `value` is the rate at position 2048 and `e2e` the per-token host protocol
    there. Per-token algorithmic bytes: all weights plus the KV rows of every position attended."""
    import torch
    q3 = _package()
    from llm_inference_b200 import checkpoint
    from llm_inference_b200.engine import DeviceWeights, Engine
    if args.gpus != 1:
        raise SystemExit("--workload config3 runs on one GPU")
    dist = Dist(1)
    shape = checkpoint.PRESETS[MODEL]
    K, W = args.steps, args.warmup
    positions = (256, 2048, 8192)
    max_seq = max(positions) + W + 2 * K + 16
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        weights = DeviceWeights.random(shape, seed=0)
        eng = Engine(weights, batch=1, max_seq=max_seq, history_cap=4 * (W + K) + 8, stream=stream.cuda_stream,
                     megakernel=args.megakernel)
        eng.capture()
    peaks = {}
    try:
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        pass
    hbm = peaks.get("hbm_gbs", 6650.0)
    per_pos, e2e = {}, None
    weight_bytes, kvpp = eng.weight_bytes_per_step(), eng.kv_bytes_per_position()
    with ClockSampler(torch.cuda.current_device()) as clk:
        for p in positions:
            eng.fill_kv_normal(p, seed=1000 + p)
            eng.set_state([17], [p])
            eng.step(W)
            ms = timed(dist, stream.cuda_stream, lambda: eng.step(K), "decode_steps")
            tok_s = K / (ms * 1e-3)
            step_bytes = weight_bytes + kvpp * (p + W + (K + 1) / 2)
            gbs = step_bytes * tok_s / 1e9
            per_pos[str(p)] = {"tok_s": round(tok_s, 1), "ms_per_token": round(ms / K, 4),
                               "bytes_per_token": int(step_bytes), "achieved_gbs": round(gbs, 1),
                               "frac": round(gbs / hbm, 4)}
            if p == 2048:
                toks = eng.sample_argmax()
                pos0 = p + W + K
                def e2e_fn():
                    t = toks
                    for i in range(K):
                        eng.forward(t, [pos0 + i])
                        t = eng.sample_argmax()
                ms_e2e = timed(dist, stream.cuda_stream, e2e_fn, "decode_e2e")
                e2e = {"value": round(K / (ms_e2e * 1e-3), 1), "unit": "tok/s", "h2d_bytes_per_step": 8,
                       "d2h_bytes_per_step": 4}
    clocks = clk.summary()
    if q3.device_error(stream.cuda_stream) != 0:
        raise SystemExit("device error flags set during the benchmark")
    mid = per_pos["2048"]
    line = {"metric": "decode tok/s (Qwen3-4B, batch 1, greedy) at positions 256/2048/8192", "value": mid["tok_s"],
            "unit": "tok/s", "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": mid["ms_per_token"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, N(0,1) KV before each position)",
            "config": {"workload": "BASELINE config 3: Qwen3-4B random-init, batch 1, greedy decode, rates at "
                                   "positions 256, 2048 and 8192", "model": MODEL, "global_batch": 1,
                       "parallelism": "dp1", "l2": "no flush: 8.0 GB of weights per token exceed the 126 MB L2",
                       "path": "one persistent cooperative kernel per token" if args.megakernel
                       else "captured graph of per-op kernels"},
            "positions": per_pos, "clocks": clocks, "e2e": e2e, "gpu_launches": eng.launches_per_step() * K,
            "step_roofline": {"bound": "hbm", "bytes_per_step": mid["bytes_per_token"], "achieved": mid["achieved_gbs"],
                              "peak": hbm, "unit": "GB/s", "frac": mid["frac"],
                              "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback"}}
    eng.close()
    dist.close()
    return line


def run_reference(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    _package()
    sys.path.insert(0, str(ROOT / "oracle"))
    import hf_cpu
    from llm_inference_b200 import checkpoint
    shape = checkpoint.PRESETS[MODEL]
    cores = os.cpu_count() or 1
    model = hf_cpu.build(shape, threads=cores)
    cache = hf_cpu.prefilled_cache(model, 1, KV_PREFILL)
    times = hf_cpu.decode_steps(model, cache, [17], args.warmup + args.steps)
    sec = sum(times[args.warmup:])
    tok_s = args.steps / sec
    sample = (f"HF transformers Qwen3ForCausalLM bf16 on CPU (the reference's harness decode loop, "
              f"bench/hf_baseline.py:10-24), 1 sequence of the workload at KV {KV_PREFILL}, one token per step")
    return {"impl": "reference", "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, N(0,1) KV)", "config": workload_config(args.gpus),
            "cpu_baseline": {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(tok_s, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mine", "reference"], default="mine")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--megakernel", action="store_true",
                    help="config3: run each token as one persistent cooperative kernel (Q3_ENGINE_MEGAKERNEL)")
    ap.add_argument("--workload", choices=["config4", "config3"], default="config4",
                    help="config4 (default): 32 sequences per GPU at KV 4096; config3: batch 1 at 256/2048/8192")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.impl == "reference":
        line = run_reference(args)
    elif args.workload == "config3":
        line = run_config3(args)
    else:
        line = run_mine(args)
        if line is not None and args.gpus == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
