"""Sharded quantized-matmul paths over torch.distributed (one process per GPU).

Only the paths that shard naturally are partitioned; every dense decode,
verify or prefill projection runs as an independent replica per GPU.

- ``ColumnShardedLMHead``: the wide lm_head, column (N) partitioned.  Rank r
  holds weight rows [r*N/P, (r+1)*N/P) with their scales and biases, computes
  its [M, N/P] slice with the decode/prefill kernels and all-gathers the
  slices into [M, N] (NCCL over NVLink).
- ``QuantizedAllToShardedLinear`` / ``QuantizedShardedToAllLinear``: the
  tensor-parallel linears that the reference's ``fast_qmm.enable`` patches
  with their collective step kept (mlxturbo/fast_qmm.py:425-462).  The first
  shards N and needs no forward collective.  The second shards K and
  all-reduces the partial outputs.
- ``ExpertParallelSwitchGLU``: the MoE expert bank, partitioned by expert.
  Rank r owns experts [r*E/P, (r+1)*E/P), and tokens are sharded by rank.
  Each rank routes its tokens' (token, k) rows to the experts' owners with one
  all-to-all, runs its local experts through the segmented grouped GEMM,
  returns the rows with a second all-to-all, and combines them (router
  weight, top_k sum) in one kernel.  For decode-sized batches the exchange
  uses fixed-capacity slots (T*top_k rows per peer, unused slots marked with a
  padding expert id that the sort and the kernels skip): no host
  synchronisation, so the block can be captured in a CUDA graph.  Larger
  batches exchange exact split sizes first (one host synchronisation) to keep
  the wire bytes down.

The local matmul defaults to ``ops.quantized_matmul``.  Expert compute and
the combine default to the CUDA kernels.  There is no CPU path: tests of the
partitioning logic on CPU (``gloo``) pass their own ``matmul`` /
``expert_fn`` / ``combine_fn``.
"""

from __future__ import annotations

import datetime
import os
from typing import Callable

import torch
import torch.distributed as dist
from torch import nn

from . import ops

__all__ = [
    "ColumnShardedLMHead", "ExpertParallelSwitchGLU", "QuantizedAllToShardedLinear",
    "QuantizedShardedToAllLinear", "init_from_env", "shard_range",
]


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int]:
    """Join the process group described by RANK / WORLD_SIZE / MASTER_* (torchrun).

    Returns (rank, world).  With CUDA the backend is NCCL and the current
    device becomes LOCAL_RANK.  A short timeout makes a rank that never
    joins (or died between steps) end the others' next collective with an
    error instead of a hang.
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
    return rank, world


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's equal share of n (n must divide evenly)."""
    if n % world:
        raise ValueError(f"{n} does not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def _group_rank_world(group) -> tuple[int, int]:
    """(rank, world) in `group`; (0, 1) when no process group exists (one GPU)."""
    if not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _qmm(x, w, s, b, group_size, bits):
    return ops.quantized_matmul(x, w, s, b, transpose=True, group_size=group_size, bits=bits)


class _ShardedBase(nn.Module):
    def __init__(self, weight, scales, biases, bias, group_size, bits, group, matmul):
        super().__init__()
        self.group = group
        self.group_size, self.bits, self.mode = group_size, bits, "affine"
        self.register_buffer("weight", weight.contiguous())
        self.register_buffer("scales", scales.contiguous())
        self.register_buffer("biases", biases.contiguous())
        self.bias = None if bias is None else nn.Parameter(bias.contiguous(), requires_grad=False)
        self._matmul = matmul or _qmm

    def _local(self, x):
        return self._matmul(x, self.weight, self.scales, self.biases, self.group_size, self.bits)


class QuantizedAllToShardedLinear(_ShardedBase):
    """Column-parallel: x replicated, output sharded along N (no forward collective)."""

    @classmethod
    def from_full(cls, weight, scales, biases, bias=None, *, group_size=64, bits=4, group=None, matmul=None):
        rank, world = _group_rank_world(group)
        a, b = shard_range(weight.shape[0], rank, world)
        return cls(weight[a:b], scales[a:b], biases[a:b], None if bias is None else bias[a:b], group_size, bits,
                   group, matmul)

    def forward(self, x):
        y = self._local(x)
        return y if self.bias is None else y + self.bias


class QuantizedShardedToAllLinear(_ShardedBase):
    """Row-parallel: x sharded along K, partial outputs all-reduced (sum)."""

    @classmethod
    def from_full(cls, weight, scales, biases, bias=None, *, group_size=64, bits=4, group=None, matmul=None):
        rank, world = _group_rank_world(group)
        K = weight.shape[1] * 32 // bits
        a, b = shard_range(K, rank, world)
        if a % group_size:
            raise ValueError(f"K shard boundary {a} is not on a quantisation group")
        wpr = 32 // bits
        return cls(weight[:, a // wpr:b // wpr], scales[:, a // group_size:b // group_size],
                   biases[:, a // group_size:b // group_size], bias, group_size, bits, group, matmul)

    def forward(self, x):
        y = self._local(x)
        dist.all_reduce(y, group=self.group)
        return y if self.bias is None else y + self.bias


class ColumnShardedLMHead(_ShardedBase):
    """The wide lm_head, column-partitioned: local [M, N/P] slice, then all-gather.

    ``forward(x, gather=True)`` returns the full [..., N] logits on every
    rank.  ``gather=False`` returns this rank's slice (for callers that
    sample or take the top-k locally before exchanging).
    """

    @classmethod
    def from_full(cls, weight, scales, biases, bias=None, *, group_size=64, bits=8, group=None, matmul=None):
        rank, world = _group_rank_world(group)
        a, b = shard_range(weight.shape[0], rank, world)
        return cls(weight[a:b], scales[a:b], biases[a:b], None if bias is None else bias[a:b], group_size, bits,
                   group, matmul)

    @property
    def shard_rows(self) -> int:
        return self.weight.shape[0]

    def forward(self, x, gather: bool = True):
        lead = x.shape[:-1]
        M = 1
        for d in lead:
            M *= d
        y = self._local(x.reshape(M, x.shape[-1]))
        if self.bias is not None:
            y = y + self.bias
        if not gather:
            return y.reshape(*lead, -1)
        world = dist.get_world_size(self.group)
        n_local = y.shape[-1]
        parts = torch.empty((world * M, n_local), dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(parts, y.contiguous(), group=self.group)
        return parts.view(world, M, n_local).permute(1, 0, 2).reshape(*lead, world * n_local)

    def topk(self, x, k: int = 1):
        """(values, token ids) of the k largest logits per row, [..., k] each.

        Each rank takes the top k of its own slice, so only M*P*k (value, id)
        pairs cross the interconnect instead of the M*N logits, then every rank
        merges the P*k candidates.  Equal values keep the lowest token id, as a
        single-device ``argmax`` does (for k = 1 exactly; for k > 1 a tie at a
        shard's k-th value may keep either id).  k=1 is greedy sampling.
        """
        lead = x.shape[:-1]
        local = self.forward(x, gather=False).reshape(-1, self.shard_rows)  # [M, N/P]
        M = local.shape[0]
        rank, world = _group_rank_world(self.group)
        kk = min(k, local.shape[1])
        if kk == 1:  # first occurrence of the maximum, like argmax on one device
            vals, idx = local.float().max(dim=-1, keepdim=True)
        else:  # (ties at a shard's k-th value may keep either id)
            vals, idx = torch.topk(local.float(), kk, dim=-1, sorted=True)
        idx = idx.to(torch.int64) + rank * self.shard_rows
        if world > 1:
            vall = torch.empty((world * M, kk), dtype=vals.dtype, device=vals.device)
            iall = torch.empty((world * M, kk), dtype=idx.dtype, device=idx.device)
            dist.all_gather_into_tensor(vall, vals.contiguous(), group=self.group)
            dist.all_gather_into_tensor(iall, idx.contiguous(), group=self.group)
            vals = vall.view(world, M, kk).permute(1, 0, 2).reshape(M, world * kk)
            idx = iall.view(world, M, kk).permute(1, 0, 2).reshape(M, world * kk)
        # order by (value descending, id ascending); ids are unique, so the merge is exact
        order = torch.argsort(idx, dim=-1)
        vals, idx = torch.gather(vals, -1, order), torch.gather(idx, -1, order)
        top = torch.argsort(vals, dim=-1, descending=True, stable=True)[:, :k]
        return (torch.gather(vals, -1, top).reshape(*lead, -1), torch.gather(idx, -1, top).reshape(*lead, -1))

    def argmax(self, x):
        """Greedy next-token ids [...]: the first occurrence of the maximum logit.

        Each rank's lm_head kernel also reduces its slice to one key per row
        (``ops.quantized_matmul_argmax``: the max logit's order-preserving bits
        over the complemented global id), so one all-gather of M keys and a max
        finish it; the logits never leave the rank.  With a bias (added after
        the matmul) the keys are taken over the biased logits instead.
        """
        lead = x.shape[:-1]
        rank, world = _group_rank_world(self.group)
        x2 = x.reshape(-1, x.shape[-1])
        if self.bias is None and self._matmul is _qmm:
            _, key = ops.quantized_matmul_argmax(x2, self.weight, self.scales, self.biases, self.group_size,
                                                 self.bits, index_offset=rank * self.shard_rows)
        else:
            local = self.forward(x2, gather=False).float() + 0.0  # -0 ties with +0
            v, i = local.max(dim=-1)
            i = i.to(torch.int64) + rank * self.shard_rows
            u = v.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
            mono = torch.where(u >= 0x80000000, (~u) & 0xFFFFFFFF, u | 0x80000000)  # order-preserving float bits
            key = (mono << 32) | (0xFFFFFFFF - i)
        if world > 1:
            keys = torch.empty((world * key.shape[0],), dtype=torch.int64, device=key.device)
            dist.all_gather_into_tensor(keys, key.contiguous(), group=self.group)
            key = ops.max_keys(keys.view(world, -1), dim=0)
        return ops.argmax_from_keys(key).reshape(lead)


def _default_expert_fn(glu, x_rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
    """down(swiglu(gate x, up x)) of each row's (local) expert, rows in input order.

    Rows whose id is >= the local expert count are padding: their outputs are
    left unwritten and must be ignored.
    """
    from .kernels import moe_counting_sort as mcs

    n = local_ids.shape[0]
    if n == 0:
        return x_rows.new_empty((0, glu.down_proj.weight.shape[1]))
    E = glu.up_proj.weight.shape[0]
    from .moe import FUSED_GLU

    if FUSED_GLU:  # received rows: the fused gate/up launch and down, outputs back in received order
        from .kernels import moe_grouped_gemm as mgg

        routed = mgg.moe_route(local_ids, E, 1)
        if routed is not None:
            order, idx_s, row_src, inv, tables = routed
        else:
            order, idx_s, row_src, inv, _ = mcs.sort_rows(local_ids, E, 1, with_tables=False)
            tables = mgg.gather_tables(idx_s, E)
        try:
            fw, fs, fb = glu.fused_gate_up()
            g, d = glu.gate_proj, glu.down_proj
            act = mgg.gather_run(x_rows, fw, fs, fb, tables, row_src=row_src, glu=True, group_size=g.group_size,
                                 bits=g.bits)
            return mgg.gather_run(act, d.weight, d.scales, d.biases, tables, row_dst=order,
                                  group_size=d.group_size, bits=d.bits)
        except NotImplementedError:
            pass
    order, idx_s, row_src, inv, _ = mcs.sort_rows(local_ids, E, 1)
    xs = x_rows[row_src.long()].unsqueeze(1)
    up = glu.up_proj(xs, idx_s, sorted_indices=True)
    gate = glu.gate_proj(xs, idx_s, sorted_indices=True)
    out = glu.down_proj(glu.activation(up, gate), idx_s, sorted_indices=True).squeeze(1)
    return out[inv.long()]


def _default_combine_fn(back: torch.Tensor, inv: torch.Tensor, w_flat: torch.Tensor, rows: int,
                        top_k: int) -> torch.Tensor:
    from .kernels import moe_combine as mc

    return mc.combine(back, inv, w_flat, rows, top_k)


class ExpertParallelSwitchGLU(nn.Module):
    """SwitchGLU whose experts are partitioned over the process group.

    ``forward(x, idx, w)``: this rank's tokens x [T, hidden], their global
    expert ids idx [T, top_k] and router weights w [T, top_k] ->
    [T, hidden] = sum_k w[t, k] * down_e(silu(gate_e x_t) * up_e x_t).
    """

    # padded exchange while each rank's padded payload stays below this (bytes)
    CAPACITY_BYTES = int(os.environ.get("MLXTURBO_EP_CAPACITY_BYTES", str(64 << 20)))

    def __init__(self, local_glu, num_experts: int, group=None, expert_fn: Callable | None = None,
                 combine_fn: Callable | None = None):
        super().__init__()
        self.glu = local_glu
        self.group = group
        self.num_experts = num_experts
        rank, world = _group_rank_world(group)
        self.experts_per_rank = num_experts // world
        if self.experts_per_rank * world != num_experts:
            raise ValueError(f"{num_experts} experts do not split evenly over {world} ranks")
        self.first_expert = rank * self.experts_per_rank
        self._expert_fn = expert_fn or _default_expert_fn
        self._combine_fn = combine_fn or _default_combine_fn

    @classmethod
    def from_full(cls, full_glu, group=None, **kw):
        """Keep this rank's slice of a full SwitchGLU's expert banks."""
        rank, world = _group_rank_world(group)
        E = full_glu.up_proj.weight.shape[0]
        a, b = shard_range(E, rank, world)
        return cls(full_glu.slice_experts(a, b), E, group, **kw)

    def forward(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        T, hidden = x.shape
        top_k = idx.shape[-1]
        _, world = _group_rank_world(self.group)
        if world == 1:  # every expert is local: no exchange
            return self.forward_local(x, idx, w)
        return self._forward_exchange(x, idx, w, T, hidden, top_k, world)

    def forward_local(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """The block with every expert of ``idx`` held by this module (one
        rank, or a whole bank on one device): no exchange."""
        T = x.shape[0]
        top_k = idx.shape[-1]
        ids32 = idx.reshape(-1).to(torch.int32)  # no copy when the router already gives int32
        if self._expert_fn is _default_expert_fn and self._combine_fn is _default_combine_fn:
            from .moe import FUSED_GLU, fused_glu_block

            if FUSED_GLU:
                y = fused_glu_block(self.glu, x, ids32, w.reshape(-1).float(), top_k)
                if y is not None:
                    return y
        rows = x[torch.arange(ids32.shape[0], device=x.device) // top_k]
        out = self._expert_fn(self.glu, rows, ids32).contiguous()
        inv = torch.arange(ids32.shape[0], dtype=torch.int32, device=x.device)
        return self._combine_fn(out, inv, w.reshape(-1).float(), T, top_k)

    def _forward_exchange(self, x, idx, w, T: int, hidden: int, top_k: int, world: int):
        ids = idx.reshape(-1).to(torch.int64)
        if world * ids.shape[0] * hidden * x.element_size() <= self.CAPACITY_BYTES:
            return self._forward_padded(x, ids, w, T, top_k, world)
        dest = ids // self.experts_per_rank
        order = torch.sort(dest, stable=True).indices  # send order: grouped by owner rank
        send_counts = torch.bincount(dest, minlength=world).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        splits = torch.stack([send_counts, recv_counts]).cpu()  # the one host sync
        send_splits, recv_splits = splits[0].tolist(), splits[1].tolist()
        n_recv = int(sum(recv_splits))
        send_x = x[(order // top_k)].contiguous()
        send_ids = (ids[order] % self.experts_per_rank).to(torch.int32)
        recv_x = x.new_empty((n_recv, hidden))
        recv_ids = torch.empty(n_recv, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_x, send_x, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_ids, send_ids, recv_splits, send_splits, group=self.group)
        out_recv = self._expert_fn(self.glu, recv_x, recv_ids).contiguous()
        back = x.new_empty((ids.shape[0], out_recv.shape[-1]))
        dist.all_to_all_single(back, out_recv, send_splits, recv_splits, group=self.group)
        inv = torch.empty_like(order)
        inv[order] = torch.arange(order.shape[0], device=order.device)
        return self._combine_fn(back, inv.to(torch.int32), w.reshape(-1).float(), T, top_k)

    def _forward_padded(self, x, ids, w, T: int, top_k: int, world: int):
        """Exchange through fixed-capacity slots: every peer gets cap = T*top_k
        rows (the most any peer can receive), unused slots carry the padding
        expert id E_local, which the counting sort and the gathered kernels
        skip.  A slot is one row of the send buffer: the token's activations
        followed by the int32 local expert id (16 bytes of tail keep rows
        16-byte aligned), so rows and ids cross in ONE all-to-all.  Equal split
        sizes: no host synchronisation, so a caller can capture the whole block
        in a CUDA graph."""
        El = self.experts_per_rank
        n = ids.shape[0]
        cap = n
        dev = x.device
        hidden = x.shape[1]
        tail = 16 // x.element_size()  # elements after each row: the id and padding
        id_cols = 4 // x.element_size()  # elements the int32 id occupies
        stride = hidden + tail
        if x.is_cuda:  # one pack launch: owner-grouped slots, local ids, token rows, padding ids
            from . import _lib

            ids32 = ops._contig(ids.to(torch.int32))
            send = x.new_empty((world * cap, stride))
            slot = torch.empty(n, dtype=torch.int32, device=dev)
            rc = _lib.load().qmm_ep_pack(ids32.data_ptr(), n, El, world, top_k, ops._contig(x).data_ptr(), hidden,
                                         send.data_ptr(), stride, slot.data_ptr(), ops._stream(dev))
            _lib.check(rc, "ep_pack")
        else:  # the same packing with torch ops (the CPU process-group tests)
            dest = ids // El
            order = torch.sort(dest, stable=True).indices
            counts = torch.zeros(world, dtype=torch.int64, device=dev).scatter_add_(0, dest, torch.ones_like(dest))
            starts = torch.cumsum(counts, 0) - counts
            pos = torch.empty_like(order)
            pos[order] = torch.arange(n, device=dev) - starts[dest[order]]
            slot = dest * cap + pos  # send-buffer row of pair i (and of its result when it comes back)
            send = x.new_zeros((world * cap, stride))
            send[slot, :hidden] = x[torch.arange(n, device=dev) // top_k]
            send_ids = send[:, hidden:hidden + id_cols].view(torch.int32)  # [world * cap, 1], a view into send
            send_ids.fill_(El)
            send_ids[slot, 0] = (ids % El).to(torch.int32)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        recv_ids = recv[:, hidden:hidden + id_cols].contiguous().view(torch.int32).reshape(-1)
        out_recv = self._expert_fn(self.glu, recv[:, :hidden], recv_ids).contiguous()  # padding rows: ignored
        back = torch.empty_like(out_recv)
        dist.all_to_all_single(back, out_recv, group=self.group)
        return self._combine_fn(back, slot.to(torch.int32), w.reshape(-1).float(), T, top_k)
