"""Python handle on the decode engine (q3_engine_* in include/q3_sm100a.h).

Mirrors the reference's Generator / Model / KVCache surface
(src/lib/inference/generator.cpp:26-63, src/lib/model/qwen3/qwen3.hpp:131-173,
src/lib/kv_cache/kv_cache.hpp:6-29): ``forward`` is Model::forward with a
host round trip, ``generate`` is Generator::generate on token ids, ``reset``
is KVCache::reset.  ``step`` is the device-resident loop used for timing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._lib import WEIGHT_FORMATS, ModelConfig, check, lib
from .config import Qwen3Config

TRACE_WORDS = 10  # Q3_TRACE_WORDS in include/q3_sm100a.h
PEER_HANDLE_BYTES = 64  # Q3_PEER_HANDLE_BYTES in include/q3_sm100a.h


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Engine:
    def __init__(self, cfg: Qwen3Config, capacity: int, device: int = 0, tp_rank: int = 0, tp_size: int = 1,
                 weights: str = "bf16"):
        """weights: "bf16" (the reference's format), "fp8" (E4M3 GEMV matrices with a
        power-of-two scale per row) or "nvfp4" (E2M1 with an E4M3 scale per 16 columns
        and a power-of-two scale per row); both quantized on the device from the BF16
        tensors."""
        if weights not in WEIGHT_FORMATS:
            raise ValueError(f"weights must be one of {sorted(WEIGHT_FORMATS)}")
        self.cfg, self.capacity, self.tp_rank, self.tp_size = cfg, capacity, tp_rank, tp_size
        self.weights = weights
        mc = ModelConfig(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.vocab,
                         int(cfg.tied), cfg.eps, cfg.theta, capacity, cfg.eos, WEIGHT_FORMATS[weights])
        h = C.c_void_p()
        check(lib().q3_engine_create(C.byref(mc), device, tp_rank, tp_size, C.byref(h)))
        self.h = h

    # ---- lifecycle
    def close(self):
        if getattr(self, "h", None):
            # batches decode on this engine's weights and stream: they go first
            for b in list(getattr(self, "_batches", ())):
                b.close()
            lib().q3_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- weights
    def init_synthetic(self, seed: int = 0):
        check(lib().q3_engine_init_synthetic(self.h, seed))

    def set_weight(self, name: str, w: np.ndarray):
        w = np.ascontiguousarray(w, dtype=np.uint16)
        rows, cols = (w.shape[0], w.shape[1]) if w.ndim == 2 else (1, w.shape[0])
        check(lib().q3_engine_set_weight(self.h, name.encode(), _ptr(w), rows, cols))

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(128)
        check(lib().q3_nccl_unique_id(buf))
        return buf.raw

    def load_safetensors(self, path) -> int:
        """Load a Hugging Face checkpoint (file, index json or directory); returns the tensor count."""
        n = C.c_size_t()
        check(lib().q3_engine_load_safetensors(self.h, os.fsencode(path), C.byref(n)))
        return int(n.value)

    def peer_handle(self) -> bytes:
        """This rank's exchange-buffer IPC handle (q3_engine_peer_handle)."""
        buf = (C.c_uint8 * PEER_HANDLE_BYTES)()
        check(lib().q3_engine_peer_handle(self.h, buf))
        return bytes(buf)

    def attach_peers(self, handles):
        """Every rank's handle in rank order (q3_engine_attach_peers)."""
        blob = b"".join(handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(lib().q3_engine_attach_peers(self.h, buf, len(handles)))

    def attach_nccl(self, uid: bytes):
        buf = C.create_string_buffer(bytes(uid), 128)
        check(lib().q3_engine_attach_nccl(self.h, buf))

    def set_comm_timeout(self, seconds: float):
        """Bound on host waits of the NCCL path (q3_engine_set_comm_timeout)."""
        check(lib().q3_engine_set_comm_timeout(self.h, float(seconds)))

    # ---- decode
    def reset(self):
        check(lib().q3_engine_reset(self.h))

    def set_tokens(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        check(lib().q3_engine_set_tokens(self.h, _ptr(ids), ids.size))

    def prefill(self, n: int):
        """Batched prefill of the next n set tokens (K/V only), q3_engine_prefill."""
        check(lib().q3_engine_prefill(self.h, n))

    def step(self, n: int = 1):
        check(lib().q3_engine_step(self.h, n))

    def sync(self):
        check(lib().q3_engine_sync(self.h))

    def forward(self, token: int) -> int:
        out = C.c_uint32()
        check(lib().q3_engine_forward(self.h, token, C.byref(out)))
        return int(out.value)

    def generate(self, prompt, max_new: int, stop_at_eos: bool = False) -> np.ndarray:
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(max(1, max_new), np.uint32)
        n = C.c_size_t()
        check(lib().q3_engine_generate(self.h, _ptr(prompt), prompt.size, max_new, int(stop_at_eos), _ptr(out),
                                       C.byref(n)))
        return out[: n.value].copy()

    def generate_text(self, tokenizer, prompt) -> bytes:
        """Generator::generate (generator.cpp:37-63) on text: the response to the
        chat-templated prompt, greedy until EOS or a full KV cache, as bytes."""
        from .tokenizer import generate_text

        return generate_text(self, tokenizer, prompt)

    # opt-in variants of the prefill (include/q3_sm100a.h, q3_engine_set_tuning)
    TUNE_FLAGS = {"tp_prefill": 0x10, "fp8_prefill": 0x20}

    @property
    def tuning(self) -> int:
        f = C.c_uint32()
        check(lib().q3_engine_tuning(self.h, C.byref(f)))
        return int(f.value)

    @tuning.setter
    def tuning(self, flags):
        """An int of Q3_TUNE_* bits, or an iterable of TUNE_FLAGS names ("all" = every flag)."""
        if not isinstance(flags, int):
            names = list(flags)
            if "all" in names:
                names = list(self.TUNE_FLAGS)
            bad = [n for n in names if n not in self.TUNE_FLAGS]
            if bad:
                raise ValueError(f"unknown tuning flag(s) {bad}; choose from {sorted(self.TUNE_FLAGS)} or 'all'")
            flags = 0
            for n in names:
                flags |= self.TUNE_FLAGS[n]
        check(lib().q3_engine_set_tuning(self.h, int(flags)))

    def trace(self, enable: bool = True):
        """Turn the launch timeline of the CUDA-graph decode path on/off."""
        ph, ct = C.c_size_t(), C.c_size_t()
        check(lib().q3_engine_trace(self.h, int(enable), None, 0, C.byref(ph), C.byref(ct)))

    def read_trace(self) -> np.ndarray:
        """[ctas, phases, TRACE_WORDS] record of the last traced step: [..., 0:2] phase (or CTA)
        start/end (globaltimer ns), [..., 2:4] clock64 there, [..., 4:8] SM cycles of parts of the
        phase, [..., 8] SM id (include/q3_sm100a.h, q3_engine_trace)."""
        ph, ct = C.c_size_t(), C.c_size_t()
        check(lib().q3_engine_trace(self.h, 1, None, 0, C.byref(ph), C.byref(ct)))
        out = np.zeros(ct.value * ph.value * TRACE_WORDS, np.uint64)
        check(lib().q3_engine_trace(self.h, 1, out.ctypes.data, out.size, C.byref(ph), C.byref(ct)))
        return out.reshape(ct.value, ph.value, -1)

    def set_position(self, pos: int):
        check(lib().q3_engine_set_position(self.h, pos))

    def fill_kv(self, upto: int, seed: int = 7):
        check(lib().q3_engine_fill_kv(self.h, upto, seed))

    # ---- state
    @property
    def position(self) -> int:
        p = C.c_size_t()
        check(lib().q3_engine_position(self.h, C.byref(p)))
        return int(p.value)

    def logits(self) -> np.ndarray:
        out = np.empty(self.cfg.vocab // self.tp_size, np.uint16)
        check(lib().q3_engine_logits(self.h, _ptr(out)))
        return out

    def argmax_history(self, n: int) -> np.ndarray:
        out = np.empty(n, np.uint32)
        check(lib().q3_engine_argmax_history(self.h, _ptr(out), n))
        return out

    def kv_slot(self, layer: int, pos: int):
        kvh = self.cfg.kv_heads // self.tp_size
        k = np.empty((kvh, 128), np.uint16)
        v = np.empty((kvh, 128), np.uint16)
        check(lib().q3_engine_kv_slot(self.h, layer, pos, _ptr(k), _ptr(v)))
        return k, v

    def kv_read(self, layer: int, pos0: int, n: int):
        """K and V slots [pos0, pos0 + n) of a layer as [n, kv_heads, 128] BF16 bits
        (the reference's KV layout; this rank's kv heads)."""
        kvh = self.cfg.kv_heads // self.tp_size
        k = np.empty((n, kvh, 128), np.uint16)
        v = np.empty((n, kvh, 128), np.uint16)
        check(lib().q3_engine_kv_read(self.h, layer, pos0, n, _ptr(k), _ptr(v)))
        return k, v

    def kv_write(self, layer: int, pos0: int, k: np.ndarray, v: np.ndarray):
        """Overwrite K and V slots [pos0, pos0 + len(k)) of a layer (reference layout)."""
        k = np.ascontiguousarray(k, dtype=np.uint16)
        v = np.ascontiguousarray(v, dtype=np.uint16)
        if k.shape != v.shape:
            raise ValueError("k and v shapes differ")
        check(lib().q3_engine_kv_write(self.h, layer, pos0, k.shape[0], _ptr(k), _ptr(v)))

    def stream(self) -> int:
        s = C.c_void_p()
        check(lib().q3_engine_stream(self.h, C.byref(s)))
        return s.value or 0

    def weight_bytes(self) -> int:
        return int(lib().q3_engine_weight_bytes(self.h))

    def kv_bytes_per_position(self) -> int:
        return int(lib().q3_engine_kv_bytes_per_position(self.h))

    def profile_step(self, kernel_class: int = 0):
        """One eager step with CUDA events around each kernel of the class
        (0 GEMVs, 1 attention, 2 all): (milliseconds, launches, bytes)."""
        ms, n, b = C.c_double(), C.c_size_t(), C.c_double()
        check(lib().q3_engine_profile_step(self.h, kernel_class, C.byref(ms), C.byref(n), C.byref(b)))
        return ms.value, int(n.value), b.value
