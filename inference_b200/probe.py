"""Fixed kernel launches for profiling under ncu.

    python -m inference_b200.probe            # GEMV then prefill GEMM
    python -m inference_b200.probe attention  # decode attention

Default: three launches of the decode GEMV (q3_gemv, Qwen3-8B gate/up shape:
24576 x 4096, 201 MB of weights) followed by three launches of the prefill
GEMM (q3_gemm, 512 tokens x 4096 -> 24576) on cuda:0, random BF16 operands.
`attention`: three launches of the paged decode attention (q3_attention_paged)
for Qwen3-8B heads (32 q / 8 kv) at position 4095 with a 16-split cluster.
"""
import torch

from .backend import B200Backend


def attention():
    qh, kvh, pos = 32, 8, 4095
    pages = pos // 64 + 1
    be = B200Backend(0)
    q = torch.randn(qh, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(pages, kvh, 64, 128, device="cuda").to(torch.bfloat16)
    v = torch.randn(pages, kvh, 64, 128, device="cuda").to(torch.bfloat16)
    table = torch.arange(pages, dtype=torch.int32, device="cuda")
    out = torch.empty(qh, 128, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        be.self_attention_paged(q, k, v, table, out, pos)
    torch.cuda.synchronize()
    print("ok")


def main():
    be = B200Backend(0)
    x = torch.randn(4096, device="cuda").to(torch.bfloat16)
    w = torch.randn(24576, 4096, device="cuda").to(torch.bfloat16)
    y = torch.empty(24576, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        be.matmul(x, w, y)
    xs = torch.randn(512, 4096, device="cuda").to(torch.bfloat16)
    ys = torch.empty(512, 24576, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        be.gemm(xs, w, ys)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    import sys

    attention() if sys.argv[1:] == ["attention"] else main()
