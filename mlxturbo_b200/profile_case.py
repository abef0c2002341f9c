"""Small, self-contained cases for ncu captures (three launches of one op).

    python -m mlxturbo_b200.profile_case qmv N K M [bits]
    python -m mlxturbo_b200.profile_case prefill M N K
"""

from __future__ import annotations

import sys

import torch

from . import ops


def main(argv: list[str]) -> None:
    kind = argv[0]
    dev = torch.device("cuda:0")
    if kind == "qmv":
        N, K, M = int(argv[1]), int(argv[2]), int(argv[3])
        bits = int(argv[4]) if len(argv) > 4 else 4
    else:
        M, N, K = int(argv[1]), int(argv[2]), int(argv[3])
        bits = 4
    wq, s, b = ops.quantize(torch.randn(N, K, device=dev) * 0.02, 64, bits)
    x = torch.randn(M, K, device=dev).bfloat16()
    for _ in range(3):
        y = ops.quantized_matmul(x, wq, s, b, bits=bits)
    torch.cuda.synchronize()
    print("ok", float(y.float().abs().mean()), ops.device_error())


if __name__ == "__main__":
    main(sys.argv[1:])
