"""Batched decode: several sequences on one engine's weights (csrc/batch.cu,
the q3_batch_* C ABI).  The reference decodes one sequence at a time
(README.md:14)."""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from ._lib import check, lib


class Batch:
    """Up to `max_seqs` sequences decoding together on `engine` (a single-GPU
    BF16 Engine), their KV pages drawn from a pool of `pool_pages` pages of 64
    positions per layer."""

    def __init__(self, engine, max_seqs: int, pool_pages: int):
        self.engine = engine
        h = C.c_void_p()
        check(lib().q3_batch_create(engine.h, max_seqs, pool_pages, C.byref(h)))
        self.h = h
        # Engine.close destroys its live batches before itself (q3_batch_destroy first)
        if not hasattr(engine, "_batches"):
            engine._batches = weakref.WeakSet()
        engine._batches.add(self)

    def close(self):
        if getattr(self, "h", None):
            lib().q3_batch_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def add(self, prompt, max_len: int = 0) -> int:
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        sid = C.c_uint32()
        check(lib().q3_batch_add(self.h, p.ctypes.data, p.size, max_len, C.byref(sid)))
        return int(sid.value)

    def fork(self, src: int) -> int:
        sid = C.c_uint32()
        check(lib().q3_batch_fork(self.h, src, C.byref(sid)))
        return int(sid.value)

    def append(self, seq: int, ids):
        a = np.ascontiguousarray(ids, dtype=np.uint32)
        check(lib().q3_batch_append(self.h, seq, a.ctypes.data, a.size))

    def release(self, seq: int):
        check(lib().q3_batch_release(self.h, seq))

    def step(self, n: int = 1):
        check(lib().q3_batch_step(self.h, n))

    def tokens(self, seq: int) -> np.ndarray:
        n = C.c_size_t()
        check(lib().q3_batch_tokens(self.h, seq, None, 0, C.byref(n)))
        out = np.zeros(n.value, np.uint32)
        check(lib().q3_batch_tokens(self.h, seq, out.ctypes.data, out.size, C.byref(n)))
        return out

    def logits(self, seq: int) -> np.ndarray:
        out = np.zeros(self.engine.cfg.vocab, np.uint16)
        check(lib().q3_batch_logits(self.h, seq, out.ctypes.data))
        return out

    def position(self, seq: int) -> int:
        p = C.c_size_t()
        check(lib().q3_batch_info(self.h, seq, C.byref(p), None))
        return int(p.value)

    @property
    def free_pages(self) -> int:
        f = C.c_size_t()
        check(lib().q3_batch_info(self.h, 0, None, C.byref(f)))
        return int(f.value)
