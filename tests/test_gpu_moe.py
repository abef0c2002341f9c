"""Parity of gather_qmm, the segmented grouped matmul and the MoE glue kernels.

Mirrors the reference's MoE gates (bench/test_moe_combine_fold.py,
moe_verify_gather._verify_v2 at moe_verify_gather.py:923-957, and the
counting sort's determinism claims, moe_counting_sort.py:41-80).
"""

import numpy as np
import pytest
import torch

import oracle as O
from _util import check_close, half_to_torch, make_weights, make_x, torch_to_half, u32_to_torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from mlxturbo_b200 import ops as _ops

    return _ops


def _bank(rng, E, N, K, gs=64, bits=4, dtype="bf16"):
    ws, ss, bs = [], [], []
    for _ in range(E):
        w, s, b = make_weights(rng, N, K, gs, bits, dtype)
        ws.append(w)
        ss.append(s)
        bs.append(b)
    return np.stack(ws), np.stack(ss), np.stack(bs)


def _route(rng, T, E, top_k, zipf=False):
    if zipf:
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        p /= p.sum()
        perm = rng.permutation(E)
        ids = [perm[rng.choice(E, top_k, replace=False, p=p)] for _ in range(T)]
    else:
        ids = [rng.choice(E, top_k, replace=False) for _ in range(T)]
    return np.stack(ids).astype(np.int32)


@pytest.mark.parametrize("T,zipf", [(1, False), (8, False), (8, True), (33, True)])
@pytest.mark.parametrize("sorted_indices", [True, False])
def test_gather_qmm_decode_widths(ops, T, zipf, sorted_indices):
    rng = np.random.default_rng(T * 7 + zipf)
    E, N, K, top_k = 24, 96, 256, 4
    w, s, b = _bank(rng, E, N, K)
    ids = _route(rng, T, E, top_k, zipf).reshape(-1)
    x = make_x(rng, T, K)
    if sorted_indices:
        order = np.argsort(ids, kind="stable")
        rhs = ids[order]
        lhs = (order // top_k).astype(np.int32)
    else:
        rhs = ids
        lhs = (np.arange(ids.size) // top_k).astype(np.int32)
    y = ops.gather_qmm(half_to_torch(x, "bf16").reshape(T, 1, K), u32_to_torch(w), half_to_torch(s, "bf16"),
                       half_to_torch(b, "bf16"), lhs_indices=torch.from_numpy(lhs).cuda(),
                       rhs_indices=torch.from_numpy(rhs).cuda(), sorted_indices=sorted_indices)
    torch.cuda.synchronize()
    assert y.shape == (rhs.size, 1, N)
    ref = O.gather_qmm(x, w, s, b, lhs, rhs)
    check_close(torch_to_half(y.reshape(-1, N)), ref, "bf16", f"T={T} zipf={zipf} sorted={sorted_indices}")


def test_gather_qmm_reference_form(ops):
    """x (rows, 1, K) already gathered, rhs sorted, no lhs (fused.py:3105-3116)."""
    rng = np.random.default_rng(2)
    E, N, K = 16, 64, 512
    w, s, b = _bank(rng, E, N, K)
    rhs = np.sort(rng.integers(0, E, size=40)).astype(np.int32)
    x = make_x(rng, 40, K)
    y = ops.gather_qmm(half_to_torch(x, "bf16").reshape(40, 1, K), u32_to_torch(w), half_to_torch(s, "bf16"),
                       half_to_torch(b, "bf16"), rhs_indices=torch.from_numpy(rhs).cuda(), sorted_indices=True)
    ref = O.gather_qmm(x, w, s, b, None, rhs)
    check_close(torch_to_half(y.reshape(40, N)), ref, "bf16", "reference form")


def test_gather_equals_dense_slice(ops):
    """The segmented gather equals dense qmm on its expert's slice, bit for bit."""
    rng = np.random.default_rng(4)
    E, N, K = 8, 128, 512
    w, s, b = _bank(rng, E, N, K)
    rhs = np.array([3] * 5 + [6] * 2, dtype=np.int32)
    x = make_x(rng, 7, K)
    xt = half_to_torch(x, "bf16")
    y = ops.gather_qmm(xt.reshape(7, 1, K), u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"),
                       rhs_indices=torch.from_numpy(rhs).cuda(), sorted_indices=True).reshape(7, N)
    for e, rows in ((3, slice(0, 5)), (6, slice(5, 7))):
        d = ops.quantized_matmul(xt[rows], u32_to_torch(w[e]), half_to_torch(s[e], "bf16"),
                                 half_to_torch(b[e], "bf16"))
        assert torch.equal(y[rows], d), f"expert {e}"


def test_sort_rows_deterministic(ops):
    from mlxturbo_b200.kernels import moe_counting_sort as mcs

    rng = np.random.default_rng(6)
    E, top_k, T = 512, 10, 2048
    ids = _route(rng, T, E, top_k, zipf=True).reshape(-1).astype(np.uint32)
    ref = O.sort_rows(ids, E, top_k)
    idt = torch.from_numpy(ids.view(np.int32)).cuda()
    for _ in range(2):
        order, idx_s, row_src, inv, tables = mcs.sort_rows(idt, E, top_k)
        got = [t.cpu().numpy().view(np.uint32) for t in (order, idx_s, row_src, inv)]
        for g, r, name in zip(got, ref, ("order", "idx_s", "row_src", "inv")):
            assert np.array_equal(g, r), name
    counts = np.bincount(ids, minlength=E).astype(np.int32)
    rs, tp = O.segment_tables(counts, 32, 48)
    assert np.array_equal(tables[0].cpu().numpy(), rs)
    assert np.array_equal(tables[1].cpu().numpy(), tp)


def test_segment_tables(ops):
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    rng = np.random.default_rng(9)
    E = 512
    ids = np.sort(rng.integers(0, E, size=5000)).astype(np.int32)
    idt = torch.from_numpy(ids).cuda()
    counts = mgg.counts_from_sorted_ids(idt, E)
    assert np.array_equal(counts.cpu().numpy(), np.bincount(ids, minlength=E))
    for bm, mix in ((32, None), (16, None), (32, 48)):
        rs, tp = mgg.segment_tables(counts, bm=bm, mix_threshold=mix)
        ors, otp = O.segment_tables(np.bincount(ids, minlength=E), bm, mix)
        assert np.array_equal(rs.cpu().numpy(), ors) and np.array_equal(tp.cpu().numpy(), otp)


def test_moe_combine(ops):
    from mlxturbo_b200.kernels import moe_combine as mc

    rng = np.random.default_rng(10)
    rows, top_k, N = 37, 10, 2048
    out_sorted = O.to_half(rng.normal(0, 1, (rows * top_k, N)))
    inv = rng.permutation(rows * top_k).astype(np.uint32)
    w = rng.random(rows * top_k).astype(np.float32)
    y = mc.combine(half_to_torch(out_sorted, "bf16"), torch.from_numpy(inv.view(np.int32)).cuda(),
                   torch.from_numpy(w).cuda(), rows, top_k)
    ref_h, ref_f = O.moe_combine(out_sorted, inv, w, rows, top_k)
    got = torch_to_half(y)
    # fp32 fmas in k order then one rounding: equal to the oracle up to fma contraction
    check_close(got, ref_f, "bf16", "combine")
    assert np.mean(got == ref_h) > 0.99


def test_segmented_epilogue(ops):
    """row_src gather fold and row_dst/row_scale epilogue (moe_grouped_gemm.py:913-1065)."""
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    rng = np.random.default_rng(12)
    E, N, K, top_k, T = 12, 64, 256, 3, 9
    w, s, b = _bank(rng, E, N, K)
    ids = _route(rng, T, E, top_k).reshape(-1).astype(np.uint32)
    order, idx_s, row_src, inv = O.sort_rows(ids, E, top_k)
    x = make_x(rng, T, K)
    scale = rng.random(ids.size).astype(np.float32)
    tables = mgg.segment_tables(mgg.counts_from_sorted_ids(torch.from_numpy(idx_s.view(np.int32)).cuda(), E))
    y = mgg.qmm_segmented(half_to_torch(x, "bf16"), u32_to_torch(w), half_to_torch(s, "bf16"),
                          half_to_torch(b, "bf16"), None, tables=tables,
                          row_src=torch.from_numpy(row_src.view(np.int32)).cuda(),
                          row_dst=torch.from_numpy(order.view(np.int32)).cuda(),
                          row_scale=torch.from_numpy(scale[order]).cuda())
    ref = O.gather_qmm(x, w, s, b, row_src.astype(np.int32), idx_s.astype(np.int32))
    ref_scattered = np.empty_like(ref)
    ref_scattered[order] = ref * scale[order][:, None]
    check_close(torch_to_half(y), ref_scattered, "bf16", "segmented epilogue")


def test_dequantize_matches_reference_template(ops):
    import os

    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "dequant_ref.npz"))
    K = int(g["K"])
    for bits in (2, 3, 4, 5, 6, 8):
        y = ops.dequantize(u32_to_torch(g[f"b{bits}_words"]), half_to_torch(g[f"b{bits}_scales"], "bf16"),
                           half_to_torch(g[f"b{bits}_biases"], "bf16"), group_size=K, bits=bits)
        assert np.array_equal(torch_to_half(y), g[f"b{bits}_deq_bf16"]), f"bits={bits}"


def test_quantize_matches_oracle(ops):
    rng = np.random.default_rng(13)
    wf = rng.normal(0, 0.02, size=(64, 512)).astype(np.float32)
    for bits in (2, 3, 4, 5, 6, 8):
        for gs in (32, 64, 128):
            wq, sc, bi = ops.quantize(torch.from_numpy(wf).cuda(), gs, bits)
            owq, osc, obi = O.quantize(wf, gs, bits, "bf16")
            assert np.array_equal(wq.cpu().numpy().view(np.uint32), owq), (bits, gs)
            assert np.array_equal(torch_to_half(sc), osc) and np.array_equal(torch_to_half(bi), obi), (bits, gs)


def test_sort_rows_padding_rows_go_last(ops):
    """Ids >= E mark padding rows (the capacity slots of the expert-parallel
    exchange): they sort after every real row, in input order, with idx_s = E,
    and the segment tables and the gather ignore them."""
    from mlxturbo_b200.kernels import moe_counting_sort as mcs
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    rng = np.random.default_rng(8)
    E, M = 16, 600
    ids = rng.integers(0, E, size=M).astype(np.uint32)
    ids[rng.random(M) < 0.3] = E  # padding
    ids[5] = E + 7
    ref = O.sort_rows(ids, E, 1)
    order, idx_s, row_src, inv, _ = mcs.sort_rows(torch.from_numpy(ids.view(np.int32)).cuda(), E, 1,
                                                  with_tables=False)
    for g, r, name in zip((order, idx_s, row_src, inv), ref, ("order", "idx_s", "row_src", "inv")):
        assert np.array_equal(g.cpu().numpy().view(np.uint32), r), name
    valid = int((ids < E).sum())
    assert (idx_s[valid:].cpu().numpy() == E).all()
    # gathered matmul over the sorted rows: padding rows are skipped, real rows are right
    N, K = 64, 256
    w, s, b = (np.stack(a) for a in zip(*[make_weights(rng, N, K) for _ in range(E)]))
    x = make_x(rng, M, K)
    tables = mgg.gather_tables(idx_s, E)
    y = mgg.gather_run(half_to_torch(x, "bf16"), u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"),
                       tables, row_src=row_src)
    got = torch_to_half(y[:valid])
    so = ref[0][:valid]
    want = np.concatenate([O.qmm(x[i:i + 1], w[ids[i]], s[ids[i]], b[ids[i]]) for i in so])
    check_close(got, want, "bf16", "padding-aware gather")


@pytest.mark.parametrize("T,E,top_k,pad", [(1, 512, 10, 0.0), (8, 512, 10, 0.0), (256, 512, 10, 0.0),
                                           (37, 16, 4, 0.3), (1638, 1024, 10, 0.1), (5, 3, 2, 0.0)])
def test_moe_route_matches_sort_and_tables(ops, T, E, top_k, pad):
    """The one-launch route (sort + segment tables) returns the counting
    sort's arrays bit for bit, padding rows last, and tables on which the
    gathered matmul gives the same bits as on qmm_gather_tables' tables."""
    from mlxturbo_b200.kernels import moe_counting_sort as mcs
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    rng = np.random.default_rng(T * 7 + E)
    ids = _route(rng, T, E, top_k, zipf=T % 2 == 0).reshape(-1).astype(np.uint32)
    ids[rng.random(ids.size) < pad] = E + 3  # padding rows
    idt = torch.from_numpy(ids.view(np.int32)).cuda()
    ref = O.sort_rows(ids, E, top_k)
    routed = mgg.moe_route(idt, E, top_k)
    assert routed is not None
    order, idx_s, row_src, inv, tables = routed
    for g, r, name in zip((order, idx_s, row_src, inv), ref, ("order", "idx_s", "row_src", "inv")):
        assert np.array_equal(g.cpu().numpy().view(np.uint32), r), name
    # the gathered matmul on the route's tables equals the one on gather_tables' tables
    N, K = 64, 256
    w, s, b = (np.stack(a) for a in zip(*[make_weights(rng, N, K) for _ in range(E)]))
    x = half_to_torch(make_x(rng, T, K), "bf16")
    args = (u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"))
    y_route = mgg.gather_run(x, *args, tables, row_src=row_src)
    o2, i2, r2, _, _ = mcs.sort_rows(idt, E, top_k, with_tables=False)
    y_ref = mgg.gather_run(x, *args, mgg.gather_tables(i2, E), row_src=r2)
    valid = int((ids < E).sum())
    torch.cuda.synchronize()
    assert torch.equal(y_route[:valid], y_ref[:valid])


def test_moe_route_declines_large_batches(ops):
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    ids = torch.zeros(20000, dtype=torch.int32, device="cuda")
    assert mgg.moe_route(ids, 512, 10) is None
    assert mgg.moe_route(ids[:100], 4096, 10) is None


@pytest.mark.parametrize("T,world", [(1, 2), (7, 4), (64, 8), (256, 8)])
def test_ep_pack_matches_the_owner_grouped_packing(ops, T, world):
    """The expert-parallel send buffers from one launch (qmm_ep_pack) equal the
    stable owner-grouped packing written with torch ops: slots, local ids,
    token rows; unclaimed slots keep the padding id."""
    from mlxturbo_b200 import _lib

    rng = np.random.default_rng(T + world)
    El, top_k, hidden = 64 // world, 10 if T > 1 else 4, 256
    E = El * world
    ids = torch.from_numpy(_route(rng, T, E, min(top_k, E)).reshape(-1)).cuda()
    top_k = ids.numel() // T
    x = half_to_torch(make_x(rng, T, hidden), "bf16")
    n = ids.numel()
    stride = hidden + 8  # each send row: hidden activations, then the int32 local id
    send = torch.zeros((world * n, stride), dtype=torch.bfloat16, device="cuda")
    send[:, hidden:].fill_(-1.0)  # every id slot is written by the launch (a claimed id or the padding id)
    slot = torch.empty(n, dtype=torch.int32, device="cuda")
    rc = _lib.load().qmm_ep_pack(ids.data_ptr(), n, El, world, top_k, x.data_ptr(), hidden, send.data_ptr(), stride,
                                 slot.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    send_x = send[:, :hidden]
    send_ids = send[:, hidden:hidden + 2].contiguous().view(torch.int32).reshape(-1)
    ids64 = ids.long()
    dest = ids64 // El
    order = torch.sort(dest, stable=True).indices
    counts = torch.bincount(dest, minlength=world)
    starts = torch.cumsum(counts, 0) - counts
    pos = torch.empty_like(order)
    pos[order] = torch.arange(n, device="cuda") - starts[dest[order]]
    ref_slot = dest * n + pos
    ref_ids = torch.full((world * n,), El, dtype=torch.int32, device="cuda")
    ref_ids[ref_slot] = (ids64 % El).to(torch.int32)
    ref_x = torch.zeros_like(send_x)
    ref_x[ref_slot] = x[torch.arange(n, device="cuda") // top_k]
    torch.cuda.synchronize()
    assert torch.equal(slot.long(), ref_slot)
    assert torch.equal(send_ids, ref_ids)
    assert torch.equal(send_x, ref_x)


@pytest.mark.parametrize("glu", [False, True])
def test_gather_run_reads_rows_of_a_wider_buffer_in_place(ops, glu):
    """x rows x_stride elements apart (an expert-parallel receive buffer, each
    row followed by its int32 expert id) give the same bits as the same rows
    packed contiguously, with and without the fused SwiGLU epilogue."""
    from mlxturbo_b200.kernels import moe_grouped_gemm as mgg

    rng = np.random.default_rng(41 + glu)
    E, top_k, T, K = 16, 4, 24, 512
    N = 64
    ids = _route(rng, T, E, top_k).reshape(-1).astype(np.int32)
    idt = torch.from_numpy(ids).cuda()
    routed = mgg.moe_route(idt, E, 1)
    assert routed is not None
    order, idx_s, row_src, inv, tables = routed
    w, s, b = (np.stack(a) for a in zip(*[make_weights(rng, N, K) for _ in range(E)]))
    args = (u32_to_torch(w), half_to_torch(s, "bf16"), half_to_torch(b, "bf16"))
    rows = ids.size
    x = half_to_torch(make_x(rng, rows, K), "bf16")
    wide = torch.full((rows, K + 8), -3.0, dtype=torch.bfloat16, device="cuda")
    wide[:, :K] = x
    y_wide = mgg.gather_run(wide[:, :K], *args, tables, row_src=row_src, glu=glu)
    y_ref = mgg.gather_run(x, *args, tables, row_src=row_src, glu=glu)
    torch.cuda.synchronize()
    assert torch.equal(y_wide, y_ref)
