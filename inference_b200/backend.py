"""B200Backend: the reference's Backend operator interface
(src/lib/backend/backend.hpp:16-42) over the op-level C ABI.

Tensors are torch CUDA tensors (torch supplies device memory and the
stream: plumbing only); every op runs a kernel of libq3_sm100a.so.  Method
names, argument order, in-place and aliasing behaviour follow backend.hpp, so
tests read like the reference's testing/tests/*.cpp.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from ._lib import check, lib


def _torch():
    import torch

    return torch


def _p(t) -> int:
    return t.data_ptr()


class RopeCache:
    """backend::RopeCache (rope_cache.hpp:14-21): fp32 cos/sin [max_pos, hd/2]."""

    def __init__(self, cosine, sine):
        self.cosine, self.sine = cosine, sine


class B200Backend:
    def __init__(self, device: int = 0):
        torch = _torch()
        self.device = torch.device("cuda", device)
        self._ws = None
        self._idx = None

    def _stream(self) -> int:
        return _torch().cuda.current_stream(self.device).cuda_stream

    def make_rope_cache(self, max_position: int, head_size: int, theta: float) -> RopeCache:
        torch = _torch()
        c = np.empty((max_position, head_size // 2), np.float32)
        s = np.empty_like(c)
        check(lib().q3_rope_tables(max_position, head_size, theta, c.ctypes.data, s.ctypes.data))
        return RopeCache(torch.from_numpy(c).to(self.device), torch.from_numpy(s).to(self.device))

    # backend.hpp:26
    def embedding(self, token_id: int, weights, output):
        check(lib().q3_embedding(_p(weights), weights.shape[0], weights.shape[1], token_id, _p(output),
                                 self._stream()))

    # backend.hpp:27
    def matmul(self, input, weights, output):
        check(lib().q3_gemv(_p(input), _p(weights), _p(output), weights.shape[0], weights.shape[1], self._stream()))

    def gemm(self, x, weights, output):
        """Batched matmul of the prefill: output[m, n] = x[m, k] . weights[n, k]^T (q3_gemm)."""
        m, k = x.shape
        n = weights.shape[0]
        check(lib().q3_gemm(_p(x), _p(weights), _p(output), m, n, k, self._stream()))

    def quantize_e4m3(self, weights, q, scale, c0: int = 0, cols: int | None = None):
        """Row-wise E4M3 with power-of-two scales (q3_quantize_e4m3): q[r, :] = E4M3(weights[r, c0:c0+cols] / scale[r])."""
        rows, full = weights.shape
        cols = full - c0 if cols is None else cols
        check(lib().q3_quantize_e4m3(_p(weights), rows, full, c0, cols, _p(q), _p(scale), self._stream()))

    def pack_e4m3(self, q):
        """Row-major E4M3 [n, k] (uint8 tensor) -> the FP8 GEMV's packed layout (q3_pack_e4m3)."""
        torch = _torch()
        n, k = q.shape
        packed = torch.empty(lib().q3_e4m3_packed_bytes(n, k), dtype=torch.uint8, device=q.device)
        check(lib().q3_pack_e4m3(_p(q), n, k, _p(packed), self._stream()))
        return packed

    def gemv_e4m3(self, x, packed, scale, output):
        """output[n] = (W[n, :] . x) * scale[n], W E4M3 in the packed layout of pack_e4m3 (q3_gemv_e4m3)."""
        n, k = output.numel(), x.numel()
        check(lib().q3_gemv_e4m3(_p(x), _p(packed), _p(scale), _p(output), n, k, self._stream()))

    def quantize_nvfp4(self, weights):
        """BF16 [n, k] (device) -> (packed NVFP4 bytes in the GEMV's layout, row scales)
        (q3_quantize_nvfp4)."""
        torch = _torch()
        n, k = weights.shape
        packed = torch.empty(lib().q3_nvfp4_packed_bytes(n, k), dtype=torch.uint8, device=weights.device)
        scale = torch.empty(n, dtype=torch.float32, device=weights.device)
        check(lib().q3_quantize_nvfp4(_p(weights), n, k, _p(packed), _p(scale), self._stream()))
        return packed, scale

    def dequant_nvfp4(self, packed, scale, n: int, k: int):
        """The exact BF16 values [n, k] of a packed NVFP4 matrix (q3_dequant_nvfp4)."""
        torch = _torch()
        out = torch.empty((n, k), dtype=torch.bfloat16, device=packed.device)
        check(lib().q3_dequant_nvfp4(_p(packed), _p(scale), n, k, _p(out), self._stream()))
        return out

    def gemv_nvfp4(self, x, packed, scale, output):
        """output[n] = W[n, :] . x for a packed NVFP4 W (q3_gemv_nvfp4)."""
        n, k = output.numel(), x.numel()
        check(lib().q3_gemv_nvfp4(_p(x), _p(packed), _p(scale), _p(output), n, k, self._stream()))

    # backend.hpp:28
    def rmsnorm(self, input, weight, output, epsilon: float):
        check(lib().q3_rmsnorm(_p(input), _p(weight), _p(output), input.numel(), epsilon, self._stream()))

    # backend.hpp:29
    def rmsnorm_add(self, residual, residual_update, weight, output, epsilon: float):
        check(lib().q3_rmsnorm_add(_p(residual), _p(residual_update), _p(weight), _p(output), residual.numel(),
                                   epsilon, self._stream()))

    # backend.hpp:30
    def rope(self, values, cache: RopeCache, position: int):
        check(lib().q3_rope(_p(values), _p(cache.cosine), _p(cache.sine), values.shape[0], values.shape[1],
                            position, self._stream()))

    # backend.hpp:31; key/value are the reference KV layout [capacity, kv_heads, head_dim]
    def self_attention(self, query, key, value, output, position: int):
        torch = _torch()
        need = lib().q3_attention_workspace_bytes(query.shape[0], key.shape[1], key.shape[0])
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        check(lib().q3_attention(_p(query), _p(key), _p(value), _p(output), query.shape[0], key.shape[1],
                                 query.shape[1], position, _p(self._ws), self._ws.numel(), self._stream()))

    def self_attention_paged(self, query, k_pages, v_pages, page_table, output, position: int):
        torch = _torch()
        need = lib().q3_attention_workspace_bytes(query.shape[0], k_pages.shape[1], position + 1)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        check(lib().q3_attention_paged(_p(query), _p(k_pages), _p(v_pages), _p(page_table), _p(output),
                                       query.shape[0], k_pages.shape[1], query.shape[1], k_pages.shape[2],
                                       position, _p(self._ws), self._ws.numel(), self._stream()))

    # backend.hpp:32
    def add(self, left, right, output):
        check(lib().q3_add(_p(left), _p(right), _p(output), output.numel(), self._stream()))

    # backend.hpp:33
    def silu(self, gate, up, output):
        check(lib().q3_silu_mul(_p(gate), _p(up), _p(output), output.numel(), self._stream()))

    # backend.hpp:33-34
    def qk_norm_rope(self, query, key, q_norm, k_norm, cache: RopeCache, token_pos: int, eps: float):
        check(lib().q3_qk_norm_rope(_p(query), _p(key), _p(q_norm), _p(k_norm), _p(cache.cosine), _p(cache.sine),
                                    query.shape[0], key.shape[0], query.shape[1], token_pos, eps, self._stream()))

    # backend.hpp:35 -- synchronises to return the id, as the reference does
    def argmax(self, logits) -> int:
        torch = _torch()
        if self._idx is None:
            self._idx = torch.zeros(1, dtype=torch.int32, device=self.device)
        check(lib().q3_argmax(_p(logits), logits.numel(), _p(self._idx), self._stream()))
        return int(self._idx.item())


def fill_normal(dst, seed: int, tensor_id: int, rows: int, cols: int, row0: int = 0, col0: int = 0,
                full_cols: int | None = None, stream: int = 0):
    check(lib().q3_fill_normal(_p(dst), seed, tensor_id, rows, cols, row0, col0, full_cols or cols, cols, stream))


def prompt_ids(n: int, seed: int = 1, vocab: int = 151936) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().q3_prompt_ids(out.ctypes.data, n, seed, vocab)
    return out


def rope_tables(max_pos: int, head_dim: int = 128, theta: float = 1e6):
    c = np.empty((max_pos, head_dim // 2), np.float32)
    s = np.empty_like(c)
    check(lib().q3_rope_tables(max_pos, head_dim, theta, c.ctypes.data, s.ctypes.data))
    return c, s
