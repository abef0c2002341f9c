"""MLX quantized checkpoints: the safetensors container (pinned both ways
against the `safetensors` package when it is installed) and model-directory
loading with per-layer quantisation overrides (mlxturbo/rebit.py:96-124)."""

import json

import numpy as np
import pytest
import torch

import oracle as O
from mlxturbo_b200 import checkpoint as ck
from mlxturbo_b200.nn import QuantizedLinear, QuantizedSwitchLinear


def _quantized(rng, N, K, gs=64, bits=4):
    w, s, b = O.quantize(rng.normal(0, 0.02, size=(N, K)).astype(np.float32), gs, bits, "bf16")
    return (torch.from_numpy(w.view(np.int32)), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16))


def test_round_trip_bit_exact(tmp_path):
    rng = np.random.default_rng(0)
    w, s, b = _quantized(rng, 48, 256)
    t = {"l.weight": w, "l.scales": s, "l.biases": b, "f16": torch.randn(3, 5).half(), "f32": torch.randn(7)}
    p = str(tmp_path / "a.safetensors")
    ck.write_safetensors(p, t, metadata={"format": "mlx"}, u32=["l.weight"])
    header, base = ck.read_header(p)
    assert header["l.weight"]["dtype"] == "U32" and header["l.scales"]["dtype"] == "BF16"
    assert base % 8 == 0 and header["__metadata__"] == {"format": "mlx"}
    r = ck.read_safetensors(p)
    for k, v in t.items():
        assert r[k].dtype == v.dtype and torch.equal(r[k].view(torch.uint8), v.contiguous().view(torch.uint8)), k
    assert set(ck.read_safetensors(p, names=["f32"])) == {"f32"}
    with pytest.raises(KeyError):
        ck.read_safetensors(p, names=["missing"])


def test_pinned_against_safetensors_package(tmp_path):
    st_np = pytest.importorskip("safetensors.numpy")
    rng = np.random.default_rng(1)
    w, s, b = _quantized(rng, 32, 128)
    p = str(tmp_path / "mine.safetensors")
    ck.write_safetensors(p, {"x.weight": w, "x.scales": s.float()}, u32=["x.weight"])
    theirs = st_np.load_file(p)
    assert theirs["x.weight"].dtype == np.uint32
    assert np.array_equal(theirs["x.weight"].view(np.int32), w.numpy())
    assert np.array_equal(theirs["x.scales"], s.float().numpy())
    q = str(tmp_path / "theirs.safetensors")
    st_np.save_file({"y.weight": w.numpy().view(np.uint32), "y.f": np.arange(6, dtype=np.float16).reshape(2, 3)}, q)
    mine = ck.read_safetensors(q)
    assert torch.equal(mine["y.weight"], w) and torch.equal(mine["y.f"], torch.arange(6).half().reshape(2, 3))


def test_model_dir_with_overrides_and_expert_bank(tmp_path):
    rng = np.random.default_rng(2)
    w1, s1, b1 = _quantized(rng, 64, 512)            # default 4-bit g64
    w2, s2, b2 = _quantized(rng, 32, 256, 32, 8)     # override: 8-bit g32
    banks = [_quantized(rng, 16, 128) for _ in range(3)]
    we, se, be = (torch.stack([bk[i] for bk in banks]) for i in range(3))
    ck.write_safetensors(str(tmp_path / "model-00001.safetensors"),
                         {"m.q.weight": w1, "m.q.scales": s1, "m.q.biases": b1, "m.norm": torch.ones(4)},
                         u32=["m.q.weight"])
    ck.write_safetensors(str(tmp_path / "model-00002.safetensors"),
                         {"m.o.weight": w2, "m.o.scales": s2, "m.o.biases": b2, "m.e.weight": we, "m.e.scales": se,
                          "m.e.biases": be}, u32=["m.o.weight", "m.e.weight"])
    (tmp_path / "config.json").write_text(json.dumps(
        {"quantization": {"group_size": 64, "bits": 4, "m.o": {"group_size": 32, "bits": 8}}}))
    layers, qc = ck.load_model_dir(str(tmp_path))
    assert set(layers) == {"m.q", "m.o", "m.e"}
    assert qc.for_layer("m.o") == (32, 8) and qc.for_layer("m.q") == (64, 4)
    q, o, e = layers["m.q"], layers["m.o"], layers["m.e"]
    assert isinstance(q, QuantizedLinear) and (q.input_dims, q.output_dims, q.bits, q.group_size) == (512, 64, 4, 64)
    assert isinstance(o, QuantizedLinear) and (o.input_dims, o.bits, o.group_size) == (256, 8, 32)
    assert isinstance(e, QuantizedSwitchLinear) and e.num_experts == 3
    assert torch.equal(q.weight, w1) and torch.equal(o.scales, s2) and torch.equal(e.biases, be)


def test_shape_mismatch_is_an_error():
    rng = np.random.default_rng(3)
    w, s, b = _quantized(rng, 16, 128)
    with pytest.raises(ValueError):
        ck.load_quantized_linear({"a.weight": w, "a.scales": s, "a.biases": b}, "a", group_size=32, bits=4)
