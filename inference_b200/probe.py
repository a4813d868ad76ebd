"""Fixed kernel launches for profiling under ncu.

    python -m inference_b200.probe

Three launches of the decode GEMV (q3_gemv, Qwen3-8B gate/up shape: 24576 x
4096, 201 MB of weights) followed by three launches of the prefill GEMM
(q3_gemm, 512 tokens x 4096 -> 24576) on cuda:0, random BF16 operands.
"""
import torch

from .backend import B200Backend


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
    main()
