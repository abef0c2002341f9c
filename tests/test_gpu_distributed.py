"""The sharded paths on two GPUs over NCCL (skipped with fewer than two):
the column-sharded lm_head and the expert-parallel MoE, with the CUDA
kernels doing the local work, against the fp32 oracle.  Ranks are spawned
processes; the process group has a short timeout so a failing rank ends
its peer's next collective with an error."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from _util import check_close, half_to_torch, make_weights, make_x, torch_to_half, u32_to_torch
    from mlxturbo_b200 import distributed as D
    from mlxturbo_b200 import nn as qnn

    D.init_from_env(backend="nccl", timeout_s=60)
    try:
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(0)  # identical full weights on both ranks
        N, K = 2048, 1024
        w, s, b = make_weights(rng, N, K, 64, 8)
        head = D.ColumnShardedLMHead.from_full(u32_to_torch(w, dev), half_to_torch(s, "bf16", dev),
                                               half_to_torch(b, "bf16", dev), group_size=64, bits=8)
        for M in (1, 5, 16, 40):
            x = make_x(np.random.default_rng(M), M, K)
            xt = half_to_torch(x, "bf16", dev)
            got = head(xt)
            check_close(torch_to_half(got), O.qmm(x, w, s, b, 64, 8), "bf16", f"lm_head M={M}")
            # greedy / top-k on the shards agree with the gathered logits
            v, i = head.topk(xt, 4)
            rv, _ = torch.topk(got.float(), 4, dim=-1)
            assert torch.equal(v, rv), f"topk values M={M}"  # bf16 logits tie: compare values, then ids' logits
            assert torch.equal(torch.gather(got.float(), -1, i), v), f"topk ids M={M}"
            assert torch.equal(head.argmax(xt), got.float().argmax(-1))

        # tensor-parallel linears on the kernels (the reference's TP patch,
        # fast_qmm.py:425-462): a column-parallel projection, a row-parallel one
        # whose all-reduce joins the NCCL stream, then a decode matmul launched
        # straight after that join on the result
        from mlxturbo_b200 import fast_qmm

        K1, N1, N2 = 1024, 512, 768
        w1, s1, b1 = make_weights(rng, N1, K1)
        w2, s2, b2 = make_weights(rng, N2, N1)
        w3, s3, b3 = make_weights(rng, 256, N2)
        col = D.QuantizedAllToShardedLinear.from_full(u32_to_torch(w1, dev), half_to_torch(s1, "bf16", dev),
                                                      half_to_torch(b1, "bf16", dev), group_size=64, bits=4)
        row = D.QuantizedShardedToAllLinear.from_full(u32_to_torch(w2, dev), half_to_torch(s2, "bf16", dev),
                                                      half_to_torch(b2, "bf16", dev), group_size=64, bits=4)
        from mlxturbo_b200 import ops

        for patched in (False, True):
            if patched:
                fast_qmm.enable()
            try:
                for M in (1, 4):
                    x = make_x(np.random.default_rng(100 + M), M, K1)
                    h = col(half_to_torch(x, "bf16", dev))  # [M, N1 / world]: this rank's columns
                    y = row(h)  # all-reduced [M, N2]
                    z = ops.quantized_matmul(y, u32_to_torch(w3, dev), half_to_torch(s3, "bf16", dev),
                                             half_to_torch(b3, "bf16", dev))
                    h_ref = O.from_half(O.to_half(O.qmm(x, w1, s1, b1)))
                    y_ref = O.qmm(O.to_half(h_ref), w2, s2, b2)
                    check_close(torch_to_half(y), y_ref, "bf16", f"TP linears M={M} patched={patched}")
                    z_ref = O.qmm(torch_to_half(y), w3, s3, b3)
                    check_close(torch_to_half(z), z_ref, "bf16", f"decode after all-reduce M={M}")
            finally:
                fast_qmm.disable()

        E, hidden, inter, top_k = 8, 256, 128, 4
        full = qnn.SwitchGLU(hidden, inter, E, device=dev)
        deq = {}
        for name, (n, k) in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)),
                             ("down_proj", (hidden, inter))):
            proj = getattr(full, name)
            mats = [make_weights(rng, n, k) for _ in range(E)]
            proj.weight.copy_(u32_to_torch(np.stack([m[0] for m in mats]), dev))
            proj.scales.copy_(half_to_torch(np.stack([m[1] for m in mats]), "bf16", dev))
            proj.biases.copy_(half_to_torch(np.stack([m[2] for m in mats]), "bf16", dev))
            deq[name] = np.stack([O.dequantize(*m, k, 64, 4) for m in mats])
        ep = D.ExpertParallelSwitchGLU.from_full(full)
        tr = np.random.default_rng(50 + rank)
        for T, cap_bytes in ((1, 16 << 20), (7, 16 << 20), (32, 16 << 20), (7, 0), (32, 0)):
            D.ExpertParallelSwitchGLU.CAPACITY_BYTES = cap_bytes  # padded exchange / exact split sizes
            x = make_x(tr, T, hidden)
            idx = np.stack([tr.choice(E, top_k, replace=False) for _ in range(T)]).astype(np.int32)
            wts = tr.random((T, top_k)).astype(np.float32)
            wts /= wts.sum(-1, keepdims=True)
            got = ep(half_to_torch(x, "bf16", dev), torch.from_numpy(idx).to(dev), torch.from_numpy(wts).to(dev))
            xf = O.from_half(x)
            ref = np.zeros((T, hidden), np.float32)
            for t in range(T):
                for k in range(top_k):
                    e = idx[t, k]
                    gt, up = deq["gate_proj"][e] @ xf[t], deq["up_proj"][e] @ xf[t]
                    ref[t] += wts[t, k] * (deq["down_proj"][e] @ (gt / (1 + np.exp(-gt)) * up))
            err = np.sqrt(np.mean((got.float().cpu().numpy() - ref) ** 2)) / np.sqrt(np.mean(ref ** 2))
            assert err <= 1e-2, f"EP T={T}: rms rel {err}"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpu_sharded_paths():
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)


def _tp_worker(rank, world, port):
    """The tensor-parallel linears and the column-sharded lm_head through a real
    NCCL process group, on however many ranks run (one GPU: world 1)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist

    from _util import check_close, half_to_torch, make_weights, make_x, torch_to_half, u32_to_torch
    from mlxturbo_b200 import distributed as D
    import datetime

    from mlxturbo_b200 import fast_qmm, ops

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    try:
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(1)
        K1, N1, N2 = 1024, 512, 768
        w1, s1, b1 = make_weights(rng, N1, K1)
        w2, s2, b2 = make_weights(rng, N2, N1)
        col = D.QuantizedAllToShardedLinear.from_full(u32_to_torch(w1, dev), half_to_torch(s1, "bf16", dev),
                                                      half_to_torch(b1, "bf16", dev), group_size=64, bits=4)
        row = D.QuantizedShardedToAllLinear.from_full(u32_to_torch(w2, dev), half_to_torch(s2, "bf16", dev),
                                                      half_to_torch(b2, "bf16", dev), group_size=64, bits=4)
        for patched in (False, True):
            if patched:
                fast_qmm.enable()
            try:
                for M in (1, 5, 16):
                    x = make_x(np.random.default_rng(200 + M), M, K1)
                    y = row(col(half_to_torch(x, "bf16", dev)))
                    h_ref = O.from_half(O.to_half(O.qmm(x, w1, s1, b1)))
                    check_close(torch_to_half(y), O.qmm(O.to_half(h_ref), w2, s2, b2), "bf16",
                                f"TP linears world={world} M={M} patched={patched}")
            finally:
                fast_qmm.disable()
        # the lm_head on column shards: greedy ids from the fused keys
        w3, s3, b3 = make_weights(rng, 4096, 1024, 64, 8)
        head = D.ColumnShardedLMHead.from_full(u32_to_torch(w3, dev), half_to_torch(s3, "bf16", dev),
                                               half_to_torch(b3, "bf16", dev), group_size=64, bits=8)
        for M in (1, 4, 16):
            xt = half_to_torch(make_x(np.random.default_rng(300 + M), M, 1024), "bf16", dev)
            logits = head(xt)
            assert torch.equal(head.argmax(xt), logits.float().argmax(-1)), f"greedy M={M}"
        assert ops.device_error() == 0
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_tensor_parallel_linears_over_nccl():
    """World size = the GPUs present, at most 2 (1 on a one-GPU box)."""
    world = min(2, torch.cuda.device_count())
    mp.spawn(_tp_worker, args=(world, _free_port()), nprocs=world, join=True)
