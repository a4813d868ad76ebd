"""Qwen3 shapes of the decode workloads (Hugging Face config.json fields,
src/lib/model/qwen3/config.hpp:8-23 of the reference)."""
from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class Qwen3Config:
    name: str
    hidden: int
    inter: int
    layers: int
    q_heads: int
    kv_heads: int
    vocab: int = 151936
    head_dim: int = 128
    tied: bool = False
    eps: float = 1e-6
    theta: float = 1e6
    eos: int = 151645

    def with_layers(self, layers: int) -> "Qwen3Config":
        return replace(self, layers=layers, name=f"{self.name}-L{layers}")

    # bytes of weights read per decode step on one GPU (all layers + lm_head + norms)
    def weight_bytes(self, weights: str = "bf16") -> int:
        """Bytes one decode step streams: every matrix, the norms, one embedding row.
        weights="fp8": one byte per GEMV weight plus a 4-byte scale per matrix row;
        "nvfp4": half a byte per GEMV weight, a block scale byte per 16, a 4-byte row scale."""
        H, I = self.hidden, self.inter
        qd, kd = self.q_heads * self.head_dim, self.kv_heads * self.head_dim
        mats = self.layer_matmul_params()
        vec = 2 * H + 2 * self.head_dim
        if weights in ("fp8", "nvfp4"):
            rows = (qd + 2 * kd) + H + 2 * I + H
            per = (lambda n: n // 2 + n // 16) if weights == "nvfp4" else (lambda n: n)
            return (per(mats) + 4 * rows + 2 * vec) * self.layers + per(self.vocab * H) + 4 * self.vocab + 2 * (H + H)
        return 2 * ((mats + vec) * self.layers + self.vocab * H + H + H)

    def layer_matmul_params(self) -> int:
        """Weights of the QKV, O, gate/up and down matrices of one layer (GEMM FLOPs = 2 x tokens x this)."""
        H, I = self.hidden, self.inter
        qd, kd = self.q_heads * self.head_dim, self.kv_heads * self.head_dim
        return (qd + 2 * kd) * H + H * qd + 2 * I * H + H * I

    def kv_bytes_per_position(self) -> int:
        return self.layers * 2 * self.kv_heads * self.head_dim * 2


QWEN3_0P6B = Qwen3Config("qwen3-0.6b", hidden=1024, inter=3072, layers=28, q_heads=16, kv_heads=8, tied=True)
QWEN3_4B = Qwen3Config("qwen3-4b", hidden=2560, inter=9728, layers=36, q_heads=32, kv_heads=8, tied=True)
QWEN3_8B = Qwen3Config("qwen3-8b", hidden=4096, inter=12288, layers=36, q_heads=32, kv_heads=8, tied=False)
QWEN3_32B = Qwen3Config("qwen3-32b", hidden=5120, inter=25600, layers=64, q_heads=64, kv_heads=8, tied=False)

MODELS = {c.name: c for c in (QWEN3_0P6B, QWEN3_4B, QWEN3_8B, QWEN3_32B)}

# Decode workloads: (model, prompt tokens, context reached by greedy decode).
WORKLOADS = {
    "qwen3-0.6b-ctx1024": (QWEN3_0P6B, 16, 1024),
    "qwen3-0.6b-ctx8192": (QWEN3_0P6B, 4096, 8192),
    "qwen3-4b-ctx4096": (QWEN3_4B, 128, 4096),
    "qwen3-8b-ctx4096": (QWEN3_8B, 512, 4096),
    "qwen3-32b-ctx8192": (QWEN3_32B, 1024, 8192),
}
