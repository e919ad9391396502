"""Host side of the batched decode engine (csrc/engine.cu) and device-resident weights.

:class:`DeviceWeights` holds a model's tensors in one device buffer at 256-byte aligned
offsets -- the reference loader's layout (src/loader.cu:143-180, :313-380), where every tensor
is a pointer into one cudaMalloc'd shard -- read from a checkpoint directory or generated on
the device from a seed. :class:`Engine` owns a q3_engine: the batched run state, the captured
decode step and the device-side token loop.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import checkpoint as ckpt
from ._lib import call, load

_B = ctypes.c_void_p


class Q3Config(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_int), ("intermediate_size", ctypes.c_int), ("n_layers", ctypes.c_int),
                ("n_heads", ctypes.c_int), ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("vocab_size", ctypes.c_int), ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


class Q3LayerWeights(ctypes.Structure):
    _fields_ = [(n, _B) for n in ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "mlp_norm", "w_gate",
                                  "w_up", "w_down")]


class Q3Weights(ctypes.Structure):
    _fields_ = [("embed", _B), ("layers", ctypes.POINTER(Q3LayerWeights)), ("final_norm", _B), ("lm_head", _B)]


class Q3EngineBuffers(ctypes.Structure):
    _fields_ = [("x", _B), ("logits", _B), ("key_cache", _B), ("value_cache", _B), ("next_token", _B), ("pos", _B),
                ("out_token", _B), ("history", _B), ("step", _B), ("batch", ctypes.c_int), ("max_seq", ctypes.c_int),
                ("history_cap", ctypes.c_int), ("launches_per_step", ctypes.c_int), ("split_from", ctypes.c_int)]


def q3_config(s: ckpt.Qwen3Shape) -> Q3Config:
    return Q3Config(s.hidden_size, s.intermediate_size, s.num_hidden_layers, s.num_attention_heads,
                    s.num_key_value_heads, s.head_dim, s.vocab_size, s.rms_norm_eps, s.rope_theta)


class _DevView:
    """A device pointer as a torch tensor (through __cuda_array_interface__)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_view(ptr: int, shape, dtype: str):
    """torch tensor over device memory owned elsewhere; dtype 'bf16' or 'i32'."""
    import torch
    if dtype == "bf16":
        return torch.as_tensor(_DevView(ptr, shape, "<i2"), device="cuda").view(torch.bfloat16)
    return torch.as_tensor(_DevView(ptr, shape, "<i4"), device="cuda")


_LAYER_SUFFIX = {"attn_norm": "input_layernorm.weight", "wq": "self_attn.q_proj.weight",
                 "wk": "self_attn.k_proj.weight", "wv": "self_attn.v_proj.weight",
                 "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
                 "wo": "self_attn.o_proj.weight", "mlp_norm": "post_attention_layernorm.weight",
                 "w_gate": "mlp.gate_proj.weight", "w_up": "mlp.up_proj.weight", "w_down": "mlp.down_proj.weight"}


class DeviceWeights:
    def __init__(self, shape: ckpt.Qwen3Shape, blob, offsets: dict[str, int]):
        self.shape = shape
        self.blob = blob  # torch uint8/int16 tensor on the device that owns the memory
        self.offsets = offsets
        base = blob.data_ptr()
        self.ptr = {k: base + o for k, o in offsets.items()}

    @staticmethod
    def _layout(shape: ckpt.Qwen3Shape):
        offsets, off = {}, 0
        shapes = ckpt.tensor_shapes(shape)
        for name in sorted(shapes):
            offsets[name] = off
            off += (int(np.prod(shapes[name])) * 2 + 255) // 256 * 256
        return shapes, offsets, off

    @classmethod
    def from_tensors(cls, shape: ckpt.Qwen3Shape, tensors: dict[str, np.ndarray], device="cuda"):
        import torch
        shapes, offsets, total = cls._layout(shape)
        host = np.zeros(total // 2, np.uint16)
        for name, o in offsets.items():
            a = np.ascontiguousarray(tensors[name], np.uint16).reshape(-1)
            host[o // 2:o // 2 + a.size] = a
        blob = torch.from_numpy(host.view(np.int16)).to(device)
        return cls(shape, blob, offsets)

    @classmethod
    def from_checkpoint(cls, model_dir, device="cuda"):
        shape, tensors = ckpt.read_checkpoint(model_dir)
        return cls.from_tensors(shape, tensors, device)

    @classmethod
    def load(cls, model_dir, device="cuda", staging_bytes: int = 32 << 20, threads: int | None = None):
        """from_checkpoint's result (the same device layout, bit for bit) without its host copies.

        The reference uploads each shard with one synchronous pageable cudaMemcpy after reading
        the whole file (src/loader.cu:143-180): one host thread, and the driver's own staging
        between the page cache and the device. Here the safetensors headers are validated first
        (checkpoint_layout) and the files are memory-mapped; the tensors, cut into chunks of at
        most `staging_bytes` in file order, are dealt out to `threads` host threads. Each thread
        owns two pinned staging buffers and a stream: it copies a chunk from the mapping into one
        buffer (page-in and memcpy, with the GIL released) while the other buffer's chunk is in
        flight to the device (cudaMemcpyAsync on its stream), so several page-cache reads and the
        DMA run at once. Returns once the weights are on the device."""
        import os
        from concurrent.futures import ThreadPoolExecutor

        import torch
        shape, spans = ckpt.checkpoint_layout(model_dir)
        _, offsets, total = cls._layout(shape)
        blob = torch.zeros(total // 2, dtype=torch.int16, device=device)  # padding bytes are zero
        obj = cls(shape, blob, offsets)
        dst = blob.view(torch.uint8)
        dev = dst.device
        maps = {}
        chunks = []  # (file map, source offset, destination offset, bytes), in file order
        for name, sp in sorted(spans.items(), key=lambda kv: (str(kv[1].path), kv[1].offset)):
            if sp.path not in maps:
                maps[sp.path] = np.memmap(sp.path, dtype=np.uint8, mode="r")
            for c0 in range(0, sp.nbytes, staging_bytes):
                chunks.append((maps[sp.path], sp.offset + c0, offsets[name] + c0, min(staging_bytes, sp.nbytes - c0)))
        n_threads = max(1, min(threads or min(8, os.cpu_count() or 1), len(chunks)))
        stage_bytes = min(staging_bytes, max((c[3] for c in chunks), default=1))
        torch.cuda.current_stream(dev).synchronize()  # the zero fill is done before any copy lands

        def worker(t: int):
            stream = torch.cuda.Stream(device=dev)
            bufs = [torch.empty(stage_bytes, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
            views = [b.numpy() for b in bufs]
            done = [None, None]
            for k, (src, s0, d0, n) in enumerate(chunks[t::n_threads]):
                i = k % 2
                if done[i] is not None:
                    done[i].synchronize()  # this buffer's previous chunk has reached the device
                np.copyto(views[i][:n], src[s0:s0 + n])
                with torch.cuda.stream(stream):
                    dst[d0:d0 + n].copy_(bufs[i][:n], non_blocking=True)
                    done[i] = torch.cuda.Event()
                    done[i].record(stream)
            stream.synchronize()

        with ThreadPoolExecutor(n_threads) as ex:
            for f in [ex.submit(worker, t) for t in range(n_threads)]:
                f.result()
        return obj

    @classmethod
    def random(cls, shape: ckpt.Qwen3Shape, seed: int = 0, device="cuda"):
        """Random-init weights generated on the device (linear N(0, 0.02), norms 1 + N(0, 0.02)),
        one generator stream per tensor in sorted-name order."""
        import torch
        shapes, offsets, total = cls._layout(shape)
        blob = torch.empty(total // 2, dtype=torch.int16, device=device)
        obj = cls(shape, blob, offsets)
        stream = torch.cuda.current_stream().cuda_stream
        for i, name in enumerate(sorted(shapes)):
            n = int(np.prod(shapes[name]))
            mean = 1.0 if ckpt.is_norm(name) else 0.0
            call("q3_fill_normal_bf16", obj.ptr[name], n, seed * 1000 + i, mean, 0.02, stream)
        return obj

    def tensor(self, name):
        return device_view(self.ptr[name], ckpt.tensor_shapes(self.shape)[name], "bf16")

    def save(self, out_dir):
        """Write these weights as a checkpoint directory in the reference's layout
        (model.safetensors, config.json, generation_config.json; what src/loader.cu reads). The
        device blob comes to the host in one copy and each tensor is written from its slice."""
        import json
        import struct
        from pathlib import Path

        out = Path(out_dir)
        out.mkdir(parents=True, exist_ok=True)
        shapes = ckpt.tensor_shapes(self.shape)
        host = self.blob.view(-1).cpu().numpy().view(np.uint8)
        header, off = {}, 0
        names = sorted(shapes)
        for name in names:
            nbytes = int(np.prod(shapes[name])) * 2
            if nbytes % 16:  # the reference loader wants 16-byte aligned offsets (src/loader.cu:273-275)
                raise ValueError(f"{name}: {nbytes} bytes is not a multiple of 16")
            header[name] = {"dtype": "BF16", "shape": list(shapes[name]), "data_offsets": [off, off + nbytes]}
            off += nbytes
        hb = json.dumps(header, separators=(",", ":")).encode()
        hb += b" " * (-(len(hb) + 8) % 16)
        with open(out / "model.safetensors", "wb") as f:
            f.write(struct.pack("<Q", len(hb)))
            f.write(hb)
            for name in names:
                o = self.offsets[name]
                f.write(memoryview(host[o:o + header[name]["data_offsets"][1] - header[name]["data_offsets"][0]]))
        (out / "config.json").write_text(json.dumps(ckpt.config_json(self.shape), indent=1))
        (out / "generation_config.json").write_text(json.dumps({"eos_token_id": self.shape.eos_token_id}))
        return out

    def q3_weights(self):
        s = self.shape
        layers = (Q3LayerWeights * s.num_hidden_layers)()
        for l in range(s.num_hidden_layers):
            for field, suffix in _LAYER_SUFFIX.items():
                setattr(layers[l], field, self.ptr[f"model.layers.{l}.{suffix}"])
        embed = self.ptr["model.embed_tokens.weight"]
        lm = embed if s.tie_word_embeddings else self.ptr["lm_head.weight"]
        w = Q3Weights(embed, layers, self.ptr["model.norm.weight"], lm)
        w._keep = layers
        return w


class Engine:
    """Batched greedy decode of `batch` independent sequences (csrc/engine.cu)."""

    def __init__(self, weights: DeviceWeights, batch: int, max_seq: int, history_cap: int = 0,
                 exact_attention: bool = False, stream=None, megakernel: bool = False,
                 split_attention: bool = False):
        import torch
        load()
        self.weights = weights
        self.shape = weights.shape
        self.batch = batch
        self.max_seq = max_seq
        self.cfg = q3_config(self.shape)
        self._w = weights.q3_weights()
        if stream is None:  # a dedicated stream: graphs cannot be captured on the legacy stream
            self._own = torch.cuda.Stream()
            stream = self._own.cuda_stream
        self.stream = stream
        handle = ctypes.c_void_p()
        call("q3_engine_create", ctypes.byref(self.cfg), ctypes.byref(self._w), batch, max_seq, history_cap,
             (1 if exact_attention else 0) | (2 if megakernel else 0) | (4 if split_attention else 0), self.stream,
             ctypes.byref(handle))
        self.handle = handle
        info = Q3EngineBuffers()
        call("q3_engine_info", self.handle, ctypes.byref(info))
        self.info = info

    # ---- the reference's per-token protocol (host in, host out)
    def forward(self, tokens, positions):
        t = (ctypes.c_int * self.batch)(*[int(v) for v in tokens])
        p = (ctypes.c_int * self.batch)(*[int(v) for v in positions])
        call("q3_engine_forward", self.handle, t, p)

    def prefill(self, seq: int, tokens, start_pos: int = 0):
        """Runs sequence `seq`'s prompt `tokens` from `start_pos` in passes of up to `batch` tokens;
        afterwards its next token is the argmax after the prompt and its position follows it."""
        t = (ctypes.c_int * len(tokens))(*[int(v) for v in tokens])
        call("q3_engine_prefill", self.handle, int(seq), t, len(tokens), int(start_pos))

    def sample_argmax(self) -> list[int]:
        out = (ctypes.c_int * self.batch)()
        call("q3_engine_sample_argmax", self.handle, out)
        return list(out)

    # ---- device-resident loop
    def set_state(self, tokens, positions):
        t = (ctypes.c_int * self.batch)(*[int(v) for v in tokens])
        p = (ctypes.c_int * self.batch)(*[int(v) for v in positions])
        call("q3_engine_set_state", self.handle, t, p)

    def capture(self):
        call("q3_engine_capture", self.handle)
        call("q3_engine_info", self.handle, ctypes.byref(self.info))

    def launches_per_step(self) -> int:
        """Kernel launches of the captured step that the next step() runs."""
        call("q3_engine_info", self.handle, ctypes.byref(self.info))
        return self.info.launches_per_step

    def split_from(self) -> int:
        """Position from which a step runs the split-KV attention instead of the fused launch
        (-1: one path for every position)."""
        return self.info.split_from

    def step(self, n: int = 1):
        call("q3_engine_step", self.handle, n)

    def fill_kv_normal(self, n_positions: int, seed: int = 0):
        call("q3_engine_fill_kv_normal", self.handle, n_positions, seed)

    # ---- inspection (each waits for the engine's stream first)
    def synchronize(self):
        import torch
        torch.cuda.ExternalStream(self.stream).synchronize()

    def logits(self):
        self.synchronize()
        return device_view(self.info.logits, (self.batch, self.shape.vocab_size), "bf16")

    def history(self):
        self.synchronize()
        return device_view(self.info.history, (self.info.history_cap, self.batch), "i32")

    def positions(self):
        self.synchronize()
        return device_view(self.info.pos, (self.batch,), "i32")

    def weight_bytes_per_step(self) -> int:
        return load().q3_weight_bytes_per_step(ctypes.byref(self.cfg))

    def kv_bytes_per_position(self) -> int:
        return load().q3_kv_bytes_per_position(ctypes.byref(self.cfg))

    def close(self):
        if getattr(self, "handle", None):
            call("q3_engine_destroy", self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
