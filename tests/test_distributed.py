"""Partitioning logic of the sharded paths on CPU: world_size-2 ``gloo`` ranks
spawned as processes.  The local quantized matmul and expert compute are
CPU stand-ins built on the oracle's dequantiser (the CUDA kernels have their
own parity tests); what is checked here is the sharding, the all-gather /
all-reduce / all-to-all plumbing and the combine order, against an
unsharded computation of the same stand-ins."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bits16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _deq(w: torch.Tensor, s: torch.Tensor, b: torch.Tensor, gs: int, bits: int) -> torch.Tensor:
    K = w.shape[-1] * 32 // bits
    wn = w.contiguous().numpy().view(np.uint32)
    return torch.from_numpy(O.dequantize(wn, _bits16(s), _bits16(b), K, gs, bits))


def cpu_matmul(x, w, s, b, gs, bits):
    return x.float() @ _deq(w, s, b, gs, bits).T


def cpu_expert_fn(glu, x_rows, local_ids):
    out = torch.zeros((x_rows.shape[0], glu.down_proj.weight.shape[1]))
    for i, e in enumerate(local_ids.tolist()):
        if e >= glu.up_proj.weight.shape[0]:  # padding row of the capacity exchange
            continue
        def proj(p, v):
            return _deq(p.weight[e], p.scales[e], p.biases[e], p.group_size, p.bits) @ v
        g = proj(glu.gate_proj, x_rows[i].float())
        u = proj(glu.up_proj, x_rows[i].float())
        out[i] = proj(glu.down_proj, torch.nn.functional.silu(g) * u)
    return out


def cpu_combine_fn(back, inv, w_flat, rows, top_k):
    picked = back[inv.long()].reshape(rows, top_k, -1)
    return (picked * w_flat.reshape(rows, top_k, 1)).sum(dim=1)


def _quantized(rng, N, K, gs=64, bits=4):
    wf = rng.normal(0, 0.02, size=(N, K)).astype(np.float32)
    w, s, b = O.quantize(wf, gs, bits, "bf16")
    return (torch.from_numpy(w.view(np.int32)), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))


def _full_glu(rng, E, hidden, inter):
    from mlxturbo_b200 import nn as qnn

    glu = qnn.SwitchGLU(hidden, inter, E)
    for name, (n, k) in (("gate_proj", (inter, hidden)), ("up_proj", (inter, hidden)), ("down_proj", (hidden, inter))):
        proj = getattr(glu, name)
        for e in range(E):
            w, s, b = _quantized(rng, n, k)
            proj.weight[e].copy_(w)
            proj.scales[e].copy_(s)
            proj.biases[e].copy_(b)
    return glu


def _worker(rank, world, port, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    from mlxturbo_b200 import distributed as D

    D.init_from_env(backend="gloo", timeout_s=60)
    try:
        rng = np.random.default_rng(0)  # the same full weights on every rank
        if case == "lm_head":
            N, K = 256, 512
            w, s, b = _quantized(rng, N, K, 64, 8)
            head = D.ColumnShardedLMHead.from_full(w, s, b, group_size=64, bits=8, matmul=cpu_matmul)
            assert head.shard_rows == N // world
            x = torch.from_numpy(np.random.default_rng(1).standard_normal((3, 2, K)).astype(np.float32))
            got = head(x)
            ref = cpu_matmul(x.reshape(6, K), w, s, b, 64, 8).reshape(3, 2, N)
            assert got.shape == (3, 2, N)
            assert torch.equal(got, ref)
            local = head(x, gather=False)
            a, z = D.shard_range(N, rank, world)
            assert torch.equal(local, ref[..., a:z])
            # sampling on the shards: only (value, id) candidates are exchanged
            for k in (1, 5):
                v, i = head.topk(x, k)
                rv, ri = torch.topk(ref, k, dim=-1)
                assert torch.equal(i, ri) and torch.equal(v, rv), k
            assert torch.equal(head.argmax(x), ref.argmax(-1))
            # ties: the lowest token id wins, as on one device
            tie = torch.zeros((1, K))
            assert int(head.argmax(tie)) == int(cpu_matmul(tie, w, s, b, 64, 8).argmax())
        elif case == "tp":
            N, K = 128, 512
            w, s, b = _quantized(rng, N, K)
            x = torch.from_numpy(np.random.default_rng(2).standard_normal((4, K)).astype(np.float32))
            ref = cpu_matmul(x, w, s, b, 64, 4)
            a2s = D.QuantizedAllToShardedLinear.from_full(w, s, b, matmul=cpu_matmul)
            a, z = D.shard_range(N, rank, world)
            assert torch.equal(a2s(x), ref[:, a:z])
            s2a = D.QuantizedShardedToAllLinear.from_full(w, s, b, matmul=cpu_matmul)
            ka, kz = D.shard_range(K, rank, world)
            torch.testing.assert_close(s2a(x[:, ka:kz].contiguous()), ref, rtol=1e-5, atol=1e-5)
        else:
            E, hidden, inter, top_k = 8, 128, 64, 3
            full = _full_glu(rng, E, hidden, inter)
            ep = D.ExpertParallelSwitchGLU.from_full(full, expert_fn=cpu_expert_fn, combine_fn=cpu_combine_fn)
            assert ep.glu.up_proj.weight.shape[0] == E // world
            tr = np.random.default_rng(10 + rank)
            cases = ((5, False), (1, False), (4, True))
            for cap_bytes in (16 << 20, 0):  # padded exchange, then exact split sizes
                D.ExpertParallelSwitchGLU.CAPACITY_BYTES = cap_bytes
                for T, skew in cases:
                    x = torch.from_numpy(tr.standard_normal((T, hidden)).astype(np.float32))
                    if skew:  # every row to rank 0's experts: rank 1 receives nothing
                        idx = np.stack([tr.choice(E // world, top_k, replace=False) for _ in range(T)])
                    else:
                        idx = np.stack([tr.choice(E, top_k, replace=False) for _ in range(T)])
                    idx = torch.from_numpy(idx.astype(np.int64))
                    wts = torch.softmax(torch.from_numpy(tr.standard_normal((T, top_k)).astype(np.float32)), -1)
                    got = ep(x, idx, wts)
                    flat = idx.reshape(-1)
                    rows = cpu_expert_fn(full, x[torch.arange(T * top_k) // top_k], flat)
                    ref = cpu_combine_fn(rows, torch.arange(T * top_k), wts.reshape(-1), T, top_k)
                    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-6)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", ["lm_head", "tp", "moe_ep"])
def test_two_rank_gloo(case):
    mp.spawn(_worker, args=(2, _free_port(), case), nprocs=2, join=True)


def test_shard_range():
    from mlxturbo_b200 import distributed as D

    assert D.shard_range(248320, 3, 8) == (93120, 124160)
    with pytest.raises(ValueError):
        D.shard_range(10, 0, 3)
