"""Decode throughput benchmark (one JSON line on rank 0).

Headline workload: Qwen3-4B, random-init on the device from
seed 0, 32 independent sequences per GPU, every layer's KV cache pre-filled with bf16 N(0, 1) up
to position 4096, greedy decode. One step decodes one token for every sequence of the GPU.
Sequences are sharded data-parallel: each rank holds a full weight replica and its own 32
sequences, with no collective on the decode path (weak scaling).

  value  tokens/s of all ranks with everything resident on the device: the captured decode
         step replayed back to back (argmax feeds the next step on the device).
  e2e    the same through the C ABI's per-token protocol with host buffers, as the reference
         engine runs (src/forward.cu:206-236): every step copies the tokens and positions from
         pinned host memory, runs the step and copies the argmax tokens back, then syncs.

Extra keys on the same line (the other BASELINE configurations):
  strong  configuration 2 at every N: Qwen3-1.7B, 64 sequences in total (64/N per GPU), KV
          pre-filled to 2048, the whole job's tokens/s (strong scaling).
  batch1  configuration 3 (N = 1): Qwen3-4B at batch 1, tokens/s and HBM fraction at positions
          256, 2048 and 8192.
  prefill (N = 1) prompt prefill of one Qwen3-4B sequence, 2048 tokens in 256-row passes.
  dropin  (N = 1) the reference's own host program, unchanged, linked against this library,
          on its own --bench protocol (src/main.cu:110-148) with a Qwen3-4B checkpoint written
          to disk; and the load time of that checkpoint by the reference's loader (the same
          program), by DeviceWeights.load and by a plain pageable upload.

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
ATTN_TRAFFIC_SOURCE = "ncu capture of one attention launch at position 4095 (profiles/attention_traffic_qwen3-4b_b32_kv4096.md)"


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


# ---------------------------------------------------------------- shared helpers

def _peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def _hbm(peaks: dict) -> tuple[float, str]:
    if "hbm_gbs" in peaks:
        return float(peaks["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs"
    return 6650.0, "fallback (6.65 TB/s)"


# ---------------------------------------------------------------- CPU baseline

CPU_BATCH = BATCH_PER_GPU  # the reference's CPU path runs one GPU's share of the workload


def _cpu_decode(steps: int, warmup: int) -> tuple[float, int, str]:
    """The reference's CPU path (its HF transformers decode loop, bench/hf_baseline.py:10-24)
    on one GPU's share of the workload: 32 sequences of Qwen3-4B with KV caches pre-filled to
    4096, all host threads. Returns (tokens/s, cores, sample description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import hf_cpu
    from llm_inference_b200 import checkpoint
    shape = checkpoint.PRESETS[MODEL]
    cores = os.cpu_count() or 1
    model = hf_cpu.build(shape, threads=cores)
    cache = hf_cpu.prefilled_cache(model, CPU_BATCH, KV_PREFILL)
    times = hf_cpu.decode_steps(model, cache, [17 + i for i in range(CPU_BATCH)], warmup + steps)[warmup:]
    sec = sum(times)
    sample = (f"HF transformers Qwen3ForCausalLM bf16 on the host CPU (the reference harness's decode loop, "
              f"bench/hf_baseline.py:10-24), {CPU_BATCH} sequences at KV {KV_PREFILL} (one GPU's share of the "
              f"workload), {steps} decode steps after {warmup} warm-up; one host, so the value does not grow with N")
    return CPU_BATCH * steps / sec, cores, sample


def cpu_baseline(steps: int = 2) -> dict:
    tok_s, cores, sample = _cpu_decode(steps, 1)
    return {"value": round(tok_s, 3), "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample}


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
    peaks = _peaks()
    hbm, hbm_src = _hbm(peaks)
    line = None
    if dist.rank == 0:
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
                              "peak": hbm, "unit": "GB/s", "frac": round(step_gbs / hbm, 4), "peak_source": hbm_src},
        }
        line["roofline"] = kernel_roofline(eng, stream, hbm, hbm_src)
    eng.close()
    del eng
    torch.cuda.synchronize()

    strong = strong_leg(dist, args)  # every rank: the strong-scaling configuration
    if line is not None:
        line["strong"] = strong
    if n == 1 and not args.no_extra:
        line["batch1"] = batch1_leg(weights, args, hbm, hbm_src)
        line["prefill"] = prefill_leg(weights)
        line["dropin"] = dropin_leg(weights, hbm, hbm_src)
    del weights
    dist.close()
    return line


def kernel_roofline(eng, stream, hbm_peak, peak_src) -> dict:
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
            "algorithmic_bytes_per_launch": int(alg), "us_per_launch": round(ms * 1e3, 2), "peak_source": peak_src,
            # dram__bytes_read.sum + dram__bytes_write.sum of the attention kernels of one launch at
            # this shape, from an ncu capture of this exact command (profiles/)
            "traffic": ATTN_TRAFFIC_BYTES, "traffic_source": ATTN_TRAFFIC_SOURCE}


STRONG_MODEL = "qwen3-1.7b"
STRONG_SEQS = 64
STRONG_KV = 2048


def strong_leg(dist, args) -> dict | None:
    """Qwen3-1.7B random-init, 64 sequences in total with KV pre-filled
    to position 2048, sharded 64/N per GPU (strong scaling: the job is fixed, the per-GPU batch
    shrinks with N). K timed greedy steps of the captured step per rank (the configuration decodes
    256 tokens per sequence; K steps of it are the sample); value = all ranks' tokens / the
    slowest rank's time. Returns the key's dict on rank 0."""
    import numpy as np
    import torch
    q3 = _package()
    from llm_inference_b200 import checkpoint
    from llm_inference_b200.engine import DeviceWeights, Engine
    n = dist.world
    if STRONG_SEQS % n:
        return None
    B, K, W = STRONG_SEQS // n, args.steps, args.warmup
    shape = checkpoint.PRESETS[STRONG_MODEL]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        weights = DeviceWeights.random(shape, seed=0)
        eng = Engine(weights, batch=B, max_seq=STRONG_KV + W + K + 16, history_cap=W + K + 8,
                     stream=stream.cuda_stream)
        eng.fill_kv_normal(STRONG_KV, seed=2000 + dist.rank)
        rng = np.random.default_rng(100 + dist.rank)
        eng.set_state(rng.integers(0, shape.vocab_size, B).tolist(), [STRONG_KV] * B)
        eng.capture()
        eng.step(W)
    torch.cuda.synchronize()
    ms = timed(dist, stream.cuda_stream, lambda: eng.step(K), "strong_steps")
    if q3.device_error(stream.cuda_stream) != 0:
        raise SystemExit("device error flags set during the strong-scaling leg")
    step_bytes = eng.weight_bytes_per_step() + B * eng.kv_bytes_per_position() * (STRONG_KV + W + (K + 1) / 2)
    launches = eng.launches_per_step()
    eng.close()
    del eng, weights
    torch.cuda.synchronize()
    if dist.rank != 0:
        return None
    hbm, src = _hbm(_peaks())
    gbs = step_bytes / (ms / K * 1e-3) / 1e9
    return {"workload": "BASELINE config 2: Qwen3-1.7B random-init, 64 sequences in total, KV pre-filled bf16 "
                        "N(0,1) to position 2048, greedy decode, sharded 64/N per GPU",
            "metric": "decode tok/s, whole job", "value": round(STRONG_SEQS * K / (ms * 1e-3), 1), "unit": "tok/s",
            "scaling": "strong", "n_gpus": n, "batch_per_gpu": B, "steps": K, "warmup": W,
            "ms_per_step": round(ms / K, 4), "gpu_launches_per_step": launches,
            "step_roofline": {"bound": "hbm", "bytes_per_step_per_gpu": int(step_bytes), "achieved": round(gbs, 1),
                              "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4), "peak_source": src}}


BATCH1_POSITIONS = (256, 2048, 8192)


def batch1_leg(weights, args, hbm, hbm_src, megakernel: bool = False) -> dict:
    """Qwen3-4B at batch 1, greedy decode, tokens/s at positions 256,
    2048 and 8192 (the cache before each position pre-filled with bf16 N(0, 1), standing in for
    the tokens a real decode would have written). One engine, one captured step, replayed K times
    at each position. Per-token algorithmic bytes: all weights plus the KV rows of every position
    attended. `e2e` is the per-token host protocol at position 2048."""
    import torch
    q3 = _package()
    from llm_inference_b200.engine import Engine
    K, W = args.steps, args.warmup
    max_seq = max(BATCH1_POSITIONS) + W + 2 * K + 16
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        eng = Engine(weights, batch=1, max_seq=max_seq, history_cap=4 * (W + K) + 8, stream=stream.cuda_stream,
                     megakernel=megakernel)
        eng.capture()
    per_pos, e2e = {}, None
    weight_bytes, kvpp = eng.weight_bytes_per_step(), eng.kv_bytes_per_position()
    one = Dist.__new__(Dist)  # this leg runs on one GPU: no process group
    one.pg = None
    for p in BATCH1_POSITIONS:
        eng.fill_kv_normal(p, seed=1000 + p)
        eng.set_state([17], [p])
        eng.step(W)
        launches = eng.launches_per_step()  # of the captured step the timed steps start with
        split = not megakernel and 0 <= eng.split_from() <= p + W
        ms = timed(one, stream.cuda_stream, lambda: eng.step(K), "batch1_steps")
        tok_s = K / (ms * 1e-3)
        step_bytes = weight_bytes + kvpp * (p + W + (K + 1) / 2)
        gbs = step_bytes * tok_s / 1e9
        per_pos[str(p)] = {"tok_s": round(tok_s, 1), "ms_per_token": round(ms / K, 4),
                           "bytes_per_token": int(step_bytes), "achieved_gbs": round(gbs, 1),
                           "frac": round(gbs / hbm, 4), "gpu_launches_per_token": launches,
                           "attention": "split-KV kernels" if split else
                           ("in the persistent kernel" if megakernel else "fused RoPE + attention launch")}
        if p == 2048:
            toks = eng.sample_argmax()
            pos0 = p + W + K
            def e2e_fn():
                t = toks
                for i in range(K):
                    eng.forward(t, [pos0 + i])
                    t = eng.sample_argmax()
            ms_e2e = timed(one, stream.cuda_stream, e2e_fn, "batch1_e2e")
            e2e = {"value": round(K / (ms_e2e * 1e-3), 1), "unit": "tok/s", "h2d_bytes_per_step": 8,
                   "d2h_bytes_per_step": 4}
    if q3.device_error(stream.cuda_stream) != 0:
        raise SystemExit("device error flags set during the batch-1 leg")
    eng.close()
    return {"workload": "BASELINE config 3: Qwen3-4B random-init, batch 1, greedy decode, rates at positions "
                        "256, 2048 and 8192 (KV before each position pre-filled bf16 N(0,1))",
            "path": "one persistent kernel per token" if megakernel else "captured graph of per-op kernels",
            "steps": K, "warmup": W, "positions": per_pos, "e2e_at_2048": e2e,
            "peak": hbm, "peak_source": hbm_src}


PREFILL_TOKENS = 2048
PREFILL_ROWS = 256  # measured: 64-row passes 11.3 k tok/s, 128 12.8 k, 256 13.9 k (the projections bound a pass)


def prefill_leg(weights) -> dict:
    """Prompt prefill (q3_engine_prefill) of one Qwen3-4B sequence: PREFILL_TOKENS random prompt
    tokens in passes of PREFILL_ROWS rows (tcgen05 projections with N = rows; each row attends
    causally over the sequence's cache). Timed from the host call to its return (the call waits
    for its work), after one warm-up prefill. The reference runs a prompt one token per forward
    (src/main.cu:122-124), i.e. at its decode rate."""
    import time as _t

    import numpy as np
    import torch
    from llm_inference_b200.engine import Engine
    shape = weights.shape
    eng = Engine(weights, batch=PREFILL_ROWS, max_seq=PREFILL_TOKENS + 64)
    prompt = np.random.default_rng(5).integers(0, shape.vocab_size, PREFILL_TOKENS).tolist()
    eng.prefill(0, prompt[:PREFILL_ROWS])  # warm-up
    torch.cuda.synchronize()
    t0 = _t.perf_counter()
    eng.prefill(0, prompt)
    sec = _t.perf_counter() - t0
    eng.close()
    return {"workload": f"Qwen3-4B, one sequence, {PREFILL_TOKENS} prompt tokens in passes of {PREFILL_ROWS} rows",
            "seconds": round(sec, 4), "tok_s": round(PREFILL_TOKENS / sec, 1),
            "timing": "host clock around q3_engine_prefill, which waits for its work"}


def _run_logged(cmd, timeout):
    r = subprocess.run([str(c) for c in cmd], capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"{cmd[0]} failed ({r.returncode}): {r.stderr[-1500:]}")
    return r


def dropin_leg(weights, hbm, hbm_src, steps: int = 128, runs: int = 3) -> dict:
    """The drop-in, measured the reference's way: its unchanged host program (src/main.cu,
    forward.cu, loader.cu, dump.cu) linked against libqwen3_b200.so in place of its kernels
    (llm-inference_b200/_build/dropin_engine), with the Qwen3-4B weights written to disk as a
    checkpoint in the reference's layout. The program's own --bench (src/main.cu:110-148): a
    one-token prompt, then `steps` greedy decode steps through its per-token protocol (host token
    in, graph replay, argmax, token back), `runs` timed runs after a warm-up; its printed seconds
    per run give tokens/s. Also the load time of that checkpoint: by the program's own loader
    (src/loader.cu, it prints it), by DeviceWeights.load and by a plain read-then-upload."""
    import shutil
    import tempfile

    import torch
    from llm_inference_b200.build import DROPIN
    from llm_inference_b200.engine import DeviceWeights
    if not DROPIN.exists():
        return {"unavailable": "the drop-in engine was not built (it needs the reference sources at build time)"}
    tmp = Path(tempfile.mkdtemp(prefix="q3_dropin_"))
    try:
        model = weights.save(tmp / "model")
        (tmp / "tokens.txt").write_text("17\n")
        r = _run_logged([DROPIN, model, "--tokens", tmp / "tokens.txt", "--bench", steps, "--runs", runs], 900)
        secs = [float(l.split()[3]) for l in r.stdout.splitlines() if l.startswith("run ")]
        tok_s = sorted(steps / s for s in secs)[len(secs) // 2]
        ref_load = None
        for l in r.stderr.splitlines():
            if l.startswith("loaded ") and " in " in l:
                ref_load = float(l.rsplit(" in ", 1)[1].split()[0])
        from llm_inference_b200 import _lib
        from llm_inference_b200.engine import q3_config
        cfg = q3_config(weights.shape)
        wb = _lib.load().q3_weight_bytes_per_step(ctypes.byref(cfg))
        kvpp = _lib.load().q3_kv_bytes_per_position(ctypes.byref(cfg))
        step_bytes = wb + kvpp * (1 + (steps + 1) / 2)  # positions 1 .. steps after the prompt
        gbs = step_bytes * tok_s / 1e9
        # loaders, warm page cache (the file was just written)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        fast = DeviceWeights.load(model)
        torch.cuda.synchronize()
        t_fast = time.perf_counter() - t0
        same = bool(torch.equal(fast.blob, weights.blob))
        del fast
        t0 = time.perf_counter()
        plain = DeviceWeights.from_checkpoint(model)
        torch.cuda.synchronize()
        t_plain = time.perf_counter() - t0
        del plain
        gb = sum(p.stat().st_size for p in model.glob("*.safetensors")) / 1e9
        return {"program": "the reference's src/main.cu + forward.cu + loader.cu + dump.cu, unchanged, linked "
                           "against libqwen3_b200.so", "model": MODEL, "protocol": f"--bench {steps} --runs {runs}",
                "tok_s": round(tok_s, 1), "ms_per_token": round(1e3 / tok_s, 4), "bytes_per_token": int(step_bytes),
                "achieved_gbs": round(gbs, 1), "frac": round(gbs / hbm, 4), "peak_source": hbm_src,
                "runs_s": secs,
                "load": {"checkpoint_gb": round(gb, 3), "page_cache": "warm (file just written)",
                         "reference_loader_s": ref_load, "fast_loader_s": round(t_fast, 3),
                         "plain_upload_s": round(t_plain, 3), "fast_loader_bit_identical": same}}
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def run_config3(args) -> dict | None:
    """Configuration 3 alone, as its own line (the same measurement as the `batch1` key)."""
    import torch
    _package()
    from llm_inference_b200 import checkpoint
    from llm_inference_b200.engine import DeviceWeights
    if args.gpus != 1:
        raise SystemExit("--workload config3 runs on one GPU")
    hbm, src = _hbm(_peaks())
    weights = DeviceWeights.random(checkpoint.PRESETS[MODEL], seed=0)
    torch.cuda.synchronize()
    b1 = batch1_leg(weights, args, hbm, src, megakernel=args.megakernel)
    mid = b1["positions"]["2048"]
    return {"metric": "decode tok/s (Qwen3-4B, batch 1, greedy) at positions 256/2048/8192", "value": mid["tok_s"],
            "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": mid["ms_per_token"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init weights, N(0,1) KV before each position)",
            "config": {"workload": b1["workload"], "model": MODEL, "global_batch": 1, "parallelism": "dp1",
                       "l2": "no flush: 8.0 GB of weights per token exceed the 126 MB L2", "path": b1["path"]},
            "positions": b1["positions"], "e2e": b1["e2e_at_2048"],
            "gpu_launches": mid["gpu_launches_per_token"] * args.steps,
            "step_roofline": {"bound": "hbm", "bytes_per_step": mid["bytes_per_token"], "achieved": mid["achieved_gbs"],
                              "peak": hbm, "unit": "GB/s", "frac": mid["frac"], "peak_source": src}}


def run_reference(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    _package()
    # a CPU decode step of the workload takes seconds: the sample is bounded to 3 timed steps
    tok_s, cores, sample = _cpu_decode(min(args.steps, 3), 1)
    return {"impl": "reference", "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(CPU_BATCH / tok_s * 1e3, 3),
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
    ap.add_argument("--no-extra", action="store_true", help="skip the batch1 and dropin legs")
    ap.add_argument("--megakernel", action="store_true",
                    help="config3: run each token as one persistent kernel (Q3_ENGINE_MEGAKERNEL)")
    ap.add_argument("--workload", choices=["config4", "config3"], default="config4",
                    help="config4 (default): the headline line with its extra keys; config3: batch 1 alone")
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
