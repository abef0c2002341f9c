"""Small, self-contained cases for ncu captures (three launches of one op).

    python -m mlxturbo_b200.profile_case qmv N K M [bits]
    python -m mlxturbo_b200.profile_case qmv_tc N K M [bits]   (the tcgen05 decode kernel, qmm_qmv_tc)
    python -m mlxturbo_b200.profile_case qmv_i8 N K M [bits]   (the integer-MMA decode kernel, qmm_qmv_i8)
    python -m mlxturbo_b200.profile_case prefill M N K
    python -m mlxturbo_b200.profile_case moe T [E]   (512-expert top-10 block, one GPU)
    python -m mlxturbo_b200.profile_case layer       (the benchmark's decode layer, M=1: 7 projections)
"""

from __future__ import annotations

import sys

import torch

from . import ops


def moe_case(T: int, E: int = 512) -> None:
    """Three calls of the expert-parallel SwitchGLU block (one GPU: no exchange)."""
    from . import distributed as D
    from . import nn as qnn

    dev = torch.device("cuda:0")
    hidden, inter, top_k = 2048, 512, 10
    glu = qnn.SwitchGLU(hidden, inter, E, device=dev)
    for proj, (n, k) in ((glu.gate_proj, (inter, hidden)), (glu.up_proj, (inter, hidden)),
                         (glu.down_proj, (hidden, inter))):
        wq, s, b = ops.quantize(torch.randn((E * n, k), device=dev) * 0.02, 64, 4)
        proj.weight.copy_(wq.view(E, n, -1))
        proj.scales.copy_(s.view(E, n, -1))
        proj.biases.copy_(b.view(E, n, -1))
    ep = D.ExpertParallelSwitchGLU(glu, E, None)
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    idx = torch.stack([torch.randperm(E, generator=g, device=dev)[:top_k] for _ in range(T)]).to(torch.int32)
    w = torch.softmax(torch.randn((T, top_k), device=dev), -1)
    x = torch.randn((T, hidden), device=dev).to(torch.bfloat16)
    for _ in range(3):
        y = ep(x, idx, w)
    torch.cuda.synchronize()
    print("ok", float(y.float().abs().mean()), ops.device_error())


# (N, K) of the benchmark's 27B-class decoder layer (4-bit, groups of 64)
LAYER = [(6144, 5120), (1024, 5120), (1024, 5120), (5120, 6144), (17408, 5120), (17408, 5120), (5120, 17408)]


def layer_case() -> None:
    """Three passes over the decode layer's seven projections, M=1, in order."""
    dev = torch.device("cuda:0")
    mats = []
    for N, K in LAYER:
        wq, s, b = ops.quantize(torch.randn(N, K, device=dev) * 0.02, 64, 4)
        mats.append((torch.randn(1, K, device=dev).bfloat16(), wq, s, b))
    for _ in range(3):
        for x, wq, s, b in mats:
            y = ops.quantized_matmul(x, wq, s, b, group_size=64, bits=4)
    torch.cuda.synchronize()
    print("ok", float(y.float().abs().mean()), ops.device_error())


def main(argv: list[str]) -> None:
    kind = argv[0]
    if kind == "layer":
        layer_case()
        return
    if kind == "moe":
        moe_case(int(argv[1]), int(argv[2]) if len(argv) > 2 else 512)
        return
    dev = torch.device("cuda:0")
    if kind in ("qmv", "qmv_tc", "qmv_i8"):
        N, K, M = int(argv[1]), int(argv[2]), int(argv[3])
        bits = int(argv[4]) if len(argv) > 4 else 4
    else:
        M, N, K = int(argv[1]), int(argv[2]), int(argv[3])
        bits = 4
    wq, s, b = ops.quantize(torch.randn(N, K, device=dev) * 0.02, 64, bits)
    x = torch.randn(M, K, device=dev).bfloat16()
    for _ in range(3):
        if kind == "qmv_tc":
            y = ops.qmv_tc(x, wq, s, b, bits=bits)
        elif kind == "qmv_i8":
            y = ops.qmv_i8(x, wq, s, b, bits=bits)
        else:
            y = ops.quantized_matmul(x, wq, s, b, bits=bits)
    torch.cuda.synchronize()
    print("ok", float(y.float().abs().mean()), ops.device_error())


if __name__ == "__main__":
    main(sys.argv[1:])
