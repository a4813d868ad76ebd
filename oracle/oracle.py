"""ctypes wrappers for the oracle libraries.  TEST INFRASTRUCTURE ONLY."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_u16p = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even, NaN quieted (src/lib/backend/cpu/bf16.hpp:27-41)."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((b[nan] >> 16) | 0x40).astype(np.uint16)
    return r


class ModelConfig(C.Structure):
    """Mirror of q3o_config / ref_config (same field order in both libraries)."""

    _fields_ = [("hidden", _sz), ("inter", _sz), ("layers", _sz), ("q_heads", _sz), ("kv_heads", _sz),
                ("head_dim", _sz), ("vocab", _sz), ("capacity", _sz), ("eps", C.c_float), ("theta", C.c_float),
                ("tied", C.c_int)]

    @classmethod
    def make(cls, hidden, inter, layers, q_heads, kv_heads, head_dim, vocab, capacity, eps=1e-6, theta=1e6,
             tied=True):
        return cls(hidden, inter, layers, q_heads, kv_heads, head_dim, vocab, capacity, eps, theta, int(bool(tied)))


CONFIGS = {}  # the oracle takes shapes from its caller


class Oracle:
    """The C restatement of the reference decode step (q3_oracle.c)."""

    def __init__(self, path: str | None = None):
        path = path or os.path.join(HERE, "libq3_oracle.so")
        if not os.path.exists(path):
            from .build_ref import build_oracle

            build_oracle()
        L = self.lib = C.CDLL(path)
        L.q3o_fill_normal.argtypes = [_u16p, C.c_uint64, C.c_uint64, _sz, _sz, _sz, _sz, _sz]
        L.q3o_prompt_ids.argtypes = [_u32p, _sz, C.c_uint64, C.c_uint32]
        L.q3o_rope_cache.argtypes = [_sz, _sz, C.c_float, _f32p, _f32p]
        L.q3o_embedding.argtypes = [C.c_uint32, _u16p, _u16p, _sz]
        L.q3o_gemv.argtypes = [_u16p, _u16p, _u16p, _sz, _sz]
        L.q3o_rmsnorm.argtypes = [_u16p, _u16p, _u16p, _sz, C.c_float]
        L.q3o_rmsnorm_add.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, C.c_float]
        L.q3o_qk_norm_rope.argtypes = [_u16p, _u16p, _u16p, _u16p, _f32p, _f32p, _sz, _sz, _sz, _sz, C.c_float]
        L.q3o_attention.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, _sz, _sz, _sz]
        L.q3o_silu.argtypes = [_u16p, _u16p, _u16p, _sz]
        L.q3o_add.argtypes = [_u16p, _u16p, _u16p, _sz]
        L.q3o_argmax.argtypes = [_u16p, _sz]
        L.q3o_argmax.restype = C.c_uint32
        L.q3o_model_create.argtypes = [C.POINTER(ModelConfig), C.c_uint64]
        L.q3o_model_create.restype = C.c_void_p
        L.q3o_model_destroy.argtypes = [C.c_void_p]
        L.q3o_model_forward.argtypes = [C.c_void_p, C.c_uint32]
        L.q3o_model_forward.restype = C.c_uint32
        L.q3o_model_logits.argtypes = [C.c_void_p]
        L.q3o_model_logits.restype = C.POINTER(C.c_uint16)
        L.q3o_model_set_token_count.argtypes = [C.c_void_p, _sz]
        L.q3o_model_token_count.argtypes = [C.c_void_p]
        L.q3o_model_token_count.restype = _sz
        L.q3o_model_kv_slot.argtypes = [C.c_void_p, _sz, _sz, _u16p, _u16p]
        L.q3o_model_weight.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.q3o_model_weight.restype = C.POINTER(C.c_uint16)
        L.q3o_e4m3.argtypes = [C.c_float]
        L.q3o_e4m3.restype = C.c_uint8
        L.q3o_e4m3_value.argtypes = [C.c_uint8]
        L.q3o_e4m3_value.restype = C.c_float
        L.q3o_quantize_e4m3.argtypes = [_u16p, _sz, _sz, _u8p, _f32p]
        L.q3o_model_quantize_fp8.argtypes = [C.c_void_p]
        L.q3o_e2m1.argtypes = [C.c_float]
        L.q3o_e2m1.restype = C.c_uint8
        L.q3o_e2m1_value.argtypes = [C.c_uint8]
        L.q3o_e2m1_value.restype = C.c_float
        L.q3o_quantize_nvfp4.argtypes = [_u16p, _sz, _sz, _u8p, _u8p, _f32p]
        L.q3o_model_quantize_nvfp4.argtypes = [C.c_void_p]

    # -- synthetic inputs
    def normal(self, seed, tensor_id, rows, cols, row0=0, col0=0, full_cols=None):
        out = np.empty((rows, cols), np.uint16)
        self.lib.q3o_fill_normal(out, seed, tensor_id, rows, cols, row0, col0, full_cols or cols)
        return out

    def prompt_ids(self, n, seed=1, vocab=151936):
        out = np.empty(n, np.uint32)
        self.lib.q3o_prompt_ids(out, n, seed, vocab)
        return out

    # -- ops (inputs/outputs are uint16 arrays holding BF16 bits)
    def rope_cache(self, max_pos, head_dim=128, theta=1e6):
        c = np.empty((max_pos, head_dim // 2), np.float32)
        s = np.empty_like(c)
        self.lib.q3o_rope_cache(max_pos, head_dim, theta, c, s)
        return c, s

    def embedding(self, token, table):
        out = np.empty(table.shape[1], np.uint16)
        self.lib.q3o_embedding(token, np.ascontiguousarray(table), out, table.shape[1])
        return out

    def gemv(self, x, w):
        y = np.empty(w.shape[0], np.uint16)
        self.lib.q3o_gemv(np.ascontiguousarray(x), np.ascontiguousarray(w), y, w.shape[0], w.shape[1])
        return y

    def rmsnorm(self, x, w, eps=1e-6):
        out = np.empty_like(x)
        self.lib.q3o_rmsnorm(np.ascontiguousarray(x), np.ascontiguousarray(w), out, x.size, eps)
        return out

    def rmsnorm_add(self, res, upd, w, eps=1e-6):
        res = np.array(res, np.uint16)
        out = np.empty_like(res)
        self.lib.q3o_rmsnorm_add(res, np.ascontiguousarray(upd), np.ascontiguousarray(w), out, res.size, eps)
        return res, out

    def qk_norm_rope(self, q, k, qn, kn, pos, theta=1e6, eps=1e-6, cos_sin=None):
        q = np.array(q, np.uint16)
        k = np.array(k, np.uint16)
        hd = q.shape[1]
        c, s = cos_sin if cos_sin is not None else self.rope_cache(pos + 1, hd, theta)
        self.lib.q3o_qk_norm_rope(q, k, np.ascontiguousarray(qn), np.ascontiguousarray(kn),
                                  np.ascontiguousarray(c), np.ascontiguousarray(s), q.shape[0], k.shape[0], hd, pos,
                                  eps)
        return q, k

    def attention(self, q, kc, vc, pos):
        """q [qH, hd]; kc, vc [capacity, kvH, hd] (reference KV layout)."""
        out = np.empty_like(q)
        self.lib.q3o_attention(np.ascontiguousarray(q), np.ascontiguousarray(kc), np.ascontiguousarray(vc), out,
                               q.shape[0], kc.shape[1], q.shape[1], pos)
        return out

    def silu(self, g, u):
        out = np.empty_like(g)
        self.lib.q3o_silu(np.ascontiguousarray(g), np.ascontiguousarray(u), out, g.size)
        return out

    def add(self, a, b):
        out = np.empty_like(a)
        self.lib.q3o_add(np.ascontiguousarray(a), np.ascontiguousarray(b), out, a.size)
        return out

    def argmax(self, logits):
        return int(self.lib.q3o_argmax(np.ascontiguousarray(logits), logits.size))

    # -- FP8 E4M3 weights (row-wise power-of-two scales)
    def e4m3(self, x: float) -> int:
        return int(self.lib.q3o_e4m3(x))

    def e4m3_value(self, q: int) -> float:
        return float(self.lib.q3o_e4m3_value(q))

    def quantize_e4m3(self, w):
        """w [rows, cols] BF16 bits -> (q [rows, cols] uint8, scale [rows] float32)."""
        w = np.ascontiguousarray(w, np.uint16)
        q = np.empty(w.shape, np.uint8)
        sc = np.empty(w.shape[0], np.float32)
        self.lib.q3o_quantize_e4m3(w, w.shape[0], w.shape[1], q, sc)
        return q, sc

    # -- NVFP4 weights (E2M1, E4M3 block scales of 16 columns, power-of-two row scales)
    def e2m1(self, x: float) -> int:
        return int(self.lib.q3o_e2m1(x))

    def e2m1_value(self, q: int) -> float:
        return float(self.lib.q3o_e2m1_value(q))

    def quantize_nvfp4(self, w):
        """w [rows, cols] BF16 bits -> (q [rows, cols] E2M1 codes, block scales [rows, cols / 16]
        E4M3 codes, row scales [rows] float32)."""
        w = np.ascontiguousarray(w, np.uint16)
        q = np.empty(w.shape, np.uint8)
        bs = np.empty((w.shape[0], w.shape[1] // 16), np.uint8)
        rs = np.empty(w.shape[0], np.float32)
        self.lib.q3o_quantize_nvfp4(w, w.shape[0], w.shape[1], q, bs, rs)
        return q, bs, rs

    # -- model
    def model(self, cfg: ModelConfig, seed: int = 0) -> "OracleModel":
        return OracleModel(self, cfg, seed)


class OracleModel:
    def __init__(self, o: Oracle, cfg: ModelConfig, seed: int):
        self.o, self.cfg = o, cfg
        self.h = o.lib.q3o_model_create(C.byref(cfg), seed)

    def close(self):
        if self.h:
            self.o.lib.q3o_model_destroy(self.h)
            self.h = None

    __del__ = close

    def forward(self, token: int) -> int:
        return int(self.o.lib.q3o_model_forward(self.h, token))

    def quantize_fp8(self) -> "OracleModel":
        """Replace every GEMV matrix by its E4M3 round trip (the FP8-weight engine's model)."""
        self.o.lib.q3o_model_quantize_fp8(self.h)
        return self

    def quantize_nvfp4(self) -> "OracleModel":
        """Replace every GEMV matrix by its NVFP4 round trip (the NVFP4-weight engine's model)."""
        self.o.lib.q3o_model_quantize_nvfp4(self.h)
        return self

    def logits(self) -> np.ndarray:
        p = self.o.lib.q3o_model_logits(self.h)
        return np.ctypeslib.as_array(p, (self.cfg.vocab,)).copy()

    @property
    def token_count(self) -> int:
        return int(self.o.lib.q3o_model_token_count(self.h))

    @token_count.setter
    def token_count(self, n: int):
        self.o.lib.q3o_model_set_token_count(self.h, n)

    def kv_slot(self, layer, pos):
        kd = self.cfg.kv_heads * self.cfg.head_dim
        k = np.empty(kd, np.uint16)
        v = np.empty(kd, np.uint16)
        self.o.lib.q3o_model_kv_slot(self.h, layer, pos, k, v)
        return k.reshape(self.cfg.kv_heads, -1), v.reshape(self.cfg.kv_heads, -1)


class RefLib:
    """The reference's own backend + Qwen3 model (oracle/_ref/libref_{cpu,cuda}.so)."""

    def __init__(self, kind: str = "cpu", path: str | None = None):
        path = path or os.path.join(HERE, "_ref", f"libref_{kind}.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} not built (run oracle/build_ref.py where the reference tree exists)")
        self.kind = kind
        L = self.lib = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_rope_cache.argtypes = [_sz, _sz, C.c_float, _f32p, _f32p]
        L.ref_op_embedding.argtypes = [C.c_uint32, _u16p, _sz, _sz, _u16p]
        L.ref_op_gemv.argtypes = [_u16p, _u16p, _u16p, _sz, _sz]
        L.ref_op_rmsnorm.argtypes = [_u16p, _u16p, _u16p, _sz, C.c_float]
        L.ref_op_rmsnorm_add.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, C.c_float]
        L.ref_op_qk_norm_rope.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, C.c_float, C.c_float]
        L.ref_op_attention.argtypes = [_u16p, _u16p, _u16p, _u16p, _sz, _sz, _sz, _sz, _sz]
        L.ref_op_silu.argtypes = [_u16p, _u16p, _u16p, _sz]
        L.ref_op_add.argtypes = [_u16p, _u16p, _u16p, _sz]
        L.ref_op_argmax.argtypes = [_u16p, _sz]
        L.ref_op_argmax.restype = C.c_longlong
        L.ref_model_create.argtypes = [C.POINTER(ModelConfig), C.c_uint64]
        L.ref_model_create.restype = C.c_void_p
        L.ref_model_destroy.argtypes = [C.c_void_p]
        L.ref_model_forward.argtypes = [C.c_void_p, C.c_uint32]
        L.ref_model_forward.restype = C.c_longlong
        L.ref_model_logits.argtypes = [C.c_void_p, _u16p]
        L.ref_model_kv_slot.argtypes = [C.c_void_p, _sz, _sz, _u16p, _u16p]
        L.ref_model_set_token_count.argtypes = [C.c_void_p, _sz]
        L.ref_model_token_count.argtypes = [C.c_void_p]
        L.ref_model_token_count.restype = _sz
        L.ref_model_fill_kv.argtypes = [C.c_void_p, _sz, C.c_uint64]
        L.ref_model_kv_range.argtypes = [C.c_void_p, _sz, _sz, _sz, _u16p, _u16p, C.c_int]

    def _check(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.ref_last_error().decode())

    def rope_cache(self, max_pos, head_dim=128, theta=1e6):
        c = np.empty((max_pos, head_dim // 2), np.float32)
        s = np.empty_like(c)
        self._check(self.lib.ref_rope_cache(max_pos, head_dim, theta, c, s))
        return c, s

    def embedding(self, token, table):
        out = np.empty(table.shape[1], np.uint16)
        self._check(self.lib.ref_op_embedding(token, np.ascontiguousarray(table), table.shape[0], table.shape[1], out))
        return out

    def gemv(self, x, w):
        y = np.empty(w.shape[0], np.uint16)
        self._check(self.lib.ref_op_gemv(np.ascontiguousarray(x), np.ascontiguousarray(w), y, w.shape[0], w.shape[1]))
        return y

    def rmsnorm(self, x, w, eps=1e-6):
        out = np.empty_like(x)
        self._check(self.lib.ref_op_rmsnorm(np.ascontiguousarray(x), np.ascontiguousarray(w), out, x.size, eps))
        return out

    def rmsnorm_add(self, res, upd, w, eps=1e-6):
        res = np.array(res, np.uint16)
        out = np.empty_like(res)
        self._check(self.lib.ref_op_rmsnorm_add(res, np.ascontiguousarray(upd), np.ascontiguousarray(w), out,
                                                res.size, eps))
        return res, out

    def qk_norm_rope(self, q, k, qn, kn, pos, theta=1e6, eps=1e-6):
        q = np.array(q, np.uint16)
        k = np.array(k, np.uint16)
        self._check(self.lib.ref_op_qk_norm_rope(q, k, np.ascontiguousarray(qn), np.ascontiguousarray(kn),
                                                 q.shape[0], k.shape[0], q.shape[1], pos, theta, eps))
        return q, k

    def attention(self, q, kc, vc, pos):
        out = np.empty_like(q)
        self._check(self.lib.ref_op_attention(np.ascontiguousarray(q), np.ascontiguousarray(kc),
                                              np.ascontiguousarray(vc), out, q.shape[0], kc.shape[1], q.shape[1],
                                              kc.shape[0], pos))
        return out

    def silu(self, g, u):
        out = np.empty_like(g)
        self._check(self.lib.ref_op_silu(np.ascontiguousarray(g), np.ascontiguousarray(u), out, g.size))
        return out

    def add(self, a, b):
        out = np.empty_like(a)
        self._check(self.lib.ref_op_add(np.ascontiguousarray(a), np.ascontiguousarray(b), out, a.size))
        return out

    def argmax(self, logits):
        r = self.lib.ref_op_argmax(np.ascontiguousarray(logits), logits.size)
        if r < 0:
            raise RuntimeError(self.lib.ref_last_error().decode())
        return int(r)

    def model(self, cfg: ModelConfig, seed: int = 0) -> "RefModel":
        return RefModel(self, cfg, seed)


class RefModel:
    def __init__(self, r: RefLib, cfg: ModelConfig, seed: int):
        self.r, self.cfg = r, cfg
        self.h = r.lib.ref_model_create(C.byref(cfg), seed)
        if not self.h:
            raise RuntimeError(r.lib.ref_last_error().decode())

    def close(self):
        if self.h:
            self.r.lib.ref_model_destroy(self.h)
            self.h = None

    __del__ = close

    def forward(self, token: int) -> int:
        t = self.r.lib.ref_model_forward(self.h, token)
        if t < 0:
            raise RuntimeError(self.r.lib.ref_last_error().decode())
        return int(t)

    def logits(self) -> np.ndarray:
        out = np.empty(self.cfg.vocab, np.uint16)
        self.r._check(self.r.lib.ref_model_logits(self.h, out))
        return out

    @property
    def token_count(self) -> int:
        return int(self.r.lib.ref_model_token_count(self.h))

    @token_count.setter
    def token_count(self, n: int):
        self.r.lib.ref_model_set_token_count(self.h, n)

    def fill_kv(self, upto: int, seed: int = 7):
        self.r._check(self.r.lib.ref_model_fill_kv(self.h, upto, seed))

    def kv_slot(self, layer, pos):
        kd = self.cfg.kv_heads * self.cfg.head_dim
        k = np.empty(kd, np.uint16)
        v = np.empty(kd, np.uint16)
        self.r._check(self.r.lib.ref_model_kv_slot(self.h, layer, pos, k, v))
        return k.reshape(self.cfg.kv_heads, -1), v.reshape(self.cfg.kv_heads, -1)

    def kv_read(self, layer, pos0, n):
        """Key / value slots [pos0, pos0 + n) of a layer, [n, kv_heads, head_dim] BF16 bits."""
        k = np.empty((n, self.cfg.kv_heads, self.cfg.head_dim), np.uint16)
        v = np.empty_like(k)
        self.r._check(self.r.lib.ref_model_kv_range(self.h, layer, pos0, n, k, v, 0))
        return k, v

    def kv_write(self, layer, pos0, k, v):
        """Overwrite key / value slots [pos0, pos0 + len(k)) of a layer."""
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        self.r._check(self.r.lib.ref_model_kv_range(self.h, layer, pos0, k.shape[0], k, v, 1))
