"""The CPU oracle, pinned against the golden vectors (no GPU).

dequant_ref.npz comes from the reference's own `dequantize` template
(quantized.h:483-569 as shipped in mlxturbo/kernels/_steel_flat.py), so these
tests pin code unpacking for bits 2..8 and the s*q+b arithmetic bit for bit.
pack_ref.npz comes from the reference's numpy packer (tools/ane_quant_probe.py).
"""

import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_dequant_matches_reference_template(oracle_mod, bits):
    g = np.load(os.path.join(GOLDEN, "dequant_ref.npz"))
    K = int(g["K"])
    w, s, b = g[f"b{bits}_words"], g[f"b{bits}_scales"], g[f"b{bits}_biases"]
    got = oracle_mod.dequantize(w, s, b, K, group_size=K, bits=bits, dtype="bf16")
    ref = g[f"b{bits}_deq_f32"]
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    # The steel loader casts the fp32 value to bf16 (one RNE rounding).
    assert np.array_equal(oracle_mod.to_half(got, "bf16"), g[f"b{bits}_deq_bf16"])


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_unpack_pack_roundtrip(oracle_mod, bits):
    g = np.load(os.path.join(GOLDEN, "dequant_ref.npz"))
    K = int(g["K"])
    w = g[f"b{bits}_words"]
    codes = oracle_mod.unpack_codes(w, K, bits)
    assert codes.max() < (1 << bits)
    assert np.array_equal(oracle_mod.pack_codes(codes, bits), w)


@pytest.mark.parametrize("bits", [4, 8])
def test_pack_layout_matches_reference_packer(oracle_mod, bits):
    g = np.load(os.path.join(GOLDEN, "pack_ref.npz"))
    codes, words = g[f"b{bits}_codes"], g[f"b{bits}_words"]
    assert np.array_equal(oracle_mod.pack_codes(codes, bits), words)
    assert np.array_equal(oracle_mod.unpack_codes(words, codes.shape[1], bits), codes)


def test_half_conversions(oracle_mod):
    rng = np.random.default_rng(0)
    v = np.concatenate([rng.normal(0, 3, 1000), [0.0, -0.0, 65504.0, 1e-8, -7e-6, 3.0e38]]).astype(np.float32)
    hb = oracle_mod.to_half(v, "bf16")
    import torch

    tb = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(hb, tb)
    fin = v[np.abs(v) < 65504]
    hf = oracle_mod.to_half(fin, "f16")
    tf = torch.from_numpy(fin).to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(hf, tf)
    assert np.array_equal(oracle_mod.from_half(hf, "f16"), torch.from_numpy(tf.view(np.int16)).view(torch.float16).float().numpy())


def test_quantize_properties(oracle_mod):
    """MLX affine quantisation: codes in range and a reconstruction error of
    about half a step.  Scales and biases are rounded to bf16 after the codes
    are chosen, so the far end of an 8-bit group drifts by up to ~1 more step."""
    rng = np.random.default_rng(3)
    wf = rng.normal(0, 0.02, size=(32, 256)).astype(np.float32)
    for bits in (4, 8):
        wq, s, b = oracle_mod.quantize(wf, 64, bits, "bf16")
        codes = oracle_mod.unpack_codes(wq, 256, bits)
        assert codes.max() <= (1 << bits) - 1
        deq = oracle_mod.dequantize(wq, s, b, 256, 64, bits, "bf16")
        step = np.abs(oracle_mod.from_half(s, "bf16")).repeat(64, axis=1)
        err = np.abs(deq - wf) / step
        assert err.max() <= 2.0 and err.mean() <= 0.4


def test_qmm_oracle_matches_numpy(oracle_mod):
    rng = np.random.default_rng(5)
    M, K, N = 3, 512, 40
    x = oracle_mod.to_half(rng.normal(0, 1, (M, K)), "bf16")
    wq, s, b = oracle_mod.quantize(rng.normal(0, 0.02, (N, K)), 64, 4, "bf16")
    y = oracle_mod.qmm(x, wq, s, b, 64, 4, "bf16")
    ref = oracle_mod.from_half(x).astype(np.float64) @ oracle_mod.dequantize(wq, s, b, K, 64, 4).astype(np.float64).T
    assert np.abs(y - ref).max() < 1e-4 * max(1.0, np.abs(ref).max())
    ymlx = oracle_mod.from_half(oracle_mod.qmv_mlx_order(x, wq, s, b), "bf16")
    assert oracle_mod.normalized_max_error(ymlx, ref) < 1e-2


def test_sort_rows_and_tables(oracle_mod):
    rng = np.random.default_rng(8)
    E, top_k, T = 16, 4, 9
    ids = np.stack([rng.choice(E, top_k, replace=False) for _ in range(T)]).reshape(-1).astype(np.uint32)
    order, idx_s, row_src, inv = oracle_mod.sort_rows(ids, E, top_k)
    assert np.array_equal(order, np.argsort(ids, kind="stable"))
    assert np.array_equal(idx_s, ids[order])
    assert np.array_equal(row_src, order // top_k)
    assert np.array_equal(inv[order], np.arange(ids.size))
    counts = np.bincount(ids, minlength=E).astype(np.int32)
    rs, tp = oracle_mod.segment_tables(counts, 32, None)
    assert rs[-1] == ids.size and np.array_equal(np.diff(rs), counts)
    assert np.array_equal(np.diff(tp), (counts + 31) // 32)
    rs2, tp2 = oracle_mod.segment_tables(counts, 32, 3)
    assert np.array_equal(np.diff(tp2), np.where(counts < 3, (counts + 15) // 16, (counts + 31) // 32))


def test_moe_combine_oracle(oracle_mod):
    rng = np.random.default_rng(9)
    rows, top_k, N = 5, 3, 24
    out_sorted = oracle_mod.to_half(rng.normal(0, 1, (rows * top_k, N)))
    perm = rng.permutation(rows * top_k).astype(np.uint32)
    w = rng.random(rows * top_k).astype(np.float32)
    y, yf = oracle_mod.moe_combine(out_sorted, perm, w, rows, top_k)
    o = oracle_mod.from_half(out_sorted)
    ref = (w.reshape(rows, top_k, 1) * o[perm].reshape(rows, top_k, N)).sum(1)
    assert np.abs(yf - ref).max() < 1e-5
