"""MLX quantized checkpoints (safetensors + config.json) loaded straight into
the quantized layers, with no repacking.

``mx.quantize`` / mlx-lm ``convert`` write every quantized linear as three
tensors, ``<prefix>.weight`` (U32 [N, K*bits/32]), ``<prefix>.scales`` and
``<prefix>.biases`` (the activation dtype, [N, K/group_size]); expert banks
carry a leading expert axis.  config.json's ``"quantization"`` holds the
default ``group_size`` / ``bits`` and optional per-layer overrides keyed by
the layer prefix (how the reference's re-quantiser writes mixed bit widths,
mlxturbo/rebit.py:96-124).  The kernels consume that layout as is, so a
checkpoint's bytes are the tensors the layers hold.

The safetensors container is read here directly: an 8-byte little-endian
header length, a JSON header of ``{name: {dtype, shape, data_offsets}}`` and
the raw little-endian data.
"""

from __future__ import annotations

import json
import os
import struct
from typing import Iterable

import numpy as np
import torch

from .nn import QuantizedLinear, QuantizedSwitchLinear

# safetensors dtype -> (numpy dtype of the raw bytes, torch dtype to present)
_DTYPES = {
    "U32": (np.int32, torch.int32),  # uint32 codes carried as int32 bit patterns (torch has no CUDA uint32 math)
    "I32": (np.int32, torch.int32),
    "BF16": (np.int16, torch.bfloat16),
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
    "I64": (np.int64, torch.int64),
    "U8": (np.uint8, torch.uint8),
    "I8": (np.int8, torch.int8),
    "BOOL": (np.bool_, torch.bool),
}
_TORCH_TO_ST = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.int32: "I32",
                torch.int64: "I64", torch.uint8: "U8", torch.int8: "I8", torch.bool: "BOOL"}


def read_header(path: str) -> tuple[dict, int]:
    """(header dict, byte offset of the data section)."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
    return header, 8 + n


def read_safetensors(path: str, names: Iterable[str] | None = None, device=None) -> dict[str, torch.Tensor]:
    """Tensors of a .safetensors file (all, or `names`), on `device` (default CPU).

    U32 tensors come back as int32 tensors holding the same bits.
    """
    header, base = read_header(path)
    want = set(names) if names is not None else None
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__" or (want is not None and name not in want):
            continue
        try:
            np_dt, t_dt = _DTYPES[meta["dtype"]]
        except KeyError:
            raise NotImplementedError(f"{name}: safetensors dtype {meta['dtype']} is not supported") from None
        b0, b1 = meta["data_offsets"]
        raw = np.array(mm[base + b0:base + b1])  # copy out of the map
        arr = raw.view(np_dt).reshape(meta["shape"])
        t = torch.from_numpy(arr)
        if t_dt is torch.bfloat16:
            t = t.view(torch.bfloat16)
        out[name] = t if device is None else t.to(device)
    if want is not None and want - set(out):
        raise KeyError(f"{sorted(want - set(out))} not in {path}")
    return out


def write_safetensors(path: str, tensors: dict[str, torch.Tensor], metadata: dict[str, str] | None = None,
                      u32: Iterable[str] = ()) -> None:
    """Write tensors (CPU or CUDA) to a .safetensors file; names in `u32` are stored as U32."""
    u32 = set(u32)
    header: dict = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        if name in u32:
            if t.dtype not in (torch.int32, getattr(torch, "uint32", torch.int32)):
                raise ValueError(f"{name}: U32 needs 32-bit integer data")
            dt = "U32"
            data = t.view(torch.int32).numpy().tobytes()
        else:
            dt = _TORCH_TO_ST.get(t.dtype)
            if dt is None:
                raise NotImplementedError(f"{name}: dtype {t.dtype}")
            data = (t.view(torch.int16) if t.dtype is torch.bfloat16 else t).numpy().tobytes()
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    if metadata:
        header["__metadata__"] = dict(metadata)
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)  # keep the data section 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


class QuantConfig:
    """config.json's "quantization": default group_size/bits plus per-prefix overrides."""

    def __init__(self, quantization: dict | None):
        q = dict(quantization or {})
        self.group_size = int(q.pop("group_size", 64))
        self.bits = int(q.pop("bits", 4))
        self.mode = q.pop("mode", "affine")
        self.overrides = {k: v for k, v in q.items() if isinstance(v, dict)}

    @classmethod
    def from_model_dir(cls, model_dir: str) -> "QuantConfig":
        with open(os.path.join(model_dir, "config.json")) as f:
            cfg = json.load(f)
        return cls(cfg.get("quantization") or cfg.get("quantization_config"))

    def for_layer(self, prefix: str) -> tuple[int, int]:
        o = self.overrides.get(prefix)
        if o is None:
            return self.group_size, self.bits
        return int(o.get("group_size", self.group_size)), int(o.get("bits", self.bits))


def quantized_prefixes(tensors: dict[str, torch.Tensor]) -> list[str]:
    """Prefixes that carry a (weight, scales, biases) triple."""
    return sorted(n[: -len(".scales")] for n in tensors
                  if n.endswith(".scales") and n[: -len(".scales")] + ".weight" in tensors)


def _check(prefix: str, w: torch.Tensor, s: torch.Tensor, b: torch.Tensor, group_size: int, bits: int) -> int:
    K = w.shape[-1] * 32 // bits
    if w.shape[-1] * 32 != K * bits or K % group_size or s.shape[-1] != K // group_size or b.shape != s.shape:
        raise ValueError(f"{prefix}: weight {tuple(w.shape)} / scales {tuple(s.shape)} do not match "
                         f"bits={bits} group_size={group_size}")
    return K


def load_quantized_linear(tensors: dict[str, torch.Tensor], prefix: str, group_size: int = 64, bits: int = 4,
                          device=None) -> QuantizedLinear:
    """A QuantizedLinear from `<prefix>.weight/.scales/.biases` (+ `.bias` if present)."""
    w, s, b = tensors[f"{prefix}.weight"], tensors[f"{prefix}.scales"], tensors[f"{prefix}.biases"]
    K = _check(prefix, w, s, b, group_size, bits)
    dev = device if device is not None else w.device
    bias = tensors.get(f"{prefix}.bias")
    layer = QuantizedLinear(K, w.shape[0], bias is not None, group_size, bits, dtype=s.dtype, device=dev)
    layer.weight.copy_(w.view(torch.int32))
    layer.scales.copy_(s)
    layer.biases.copy_(b)
    if bias is not None:
        layer.bias.data.copy_(bias)
    return layer


def load_switch_linear(tensors: dict[str, torch.Tensor], prefix: str, group_size: int = 64, bits: int = 4,
                       device=None) -> QuantizedSwitchLinear:
    """A QuantizedSwitchLinear (expert bank, leading E axis) from its three tensors."""
    w, s, b = tensors[f"{prefix}.weight"], tensors[f"{prefix}.scales"], tensors[f"{prefix}.biases"]
    K = _check(prefix, w, s, b, group_size, bits)
    dev = device if device is not None else w.device
    bias = tensors.get(f"{prefix}.bias")
    layer = QuantizedSwitchLinear(K, w.shape[1], w.shape[0], bias is not None, group_size, bits, dtype=s.dtype,
                                  device=dev)
    layer.weight.copy_(w.view(torch.int32))
    layer.scales.copy_(s)
    layer.biases.copy_(b)
    if bias is not None:
        layer.bias.data.copy_(bias)
    return layer


def load_model_dir(model_dir: str, device=None) -> tuple[dict[str, torch.nn.Module], QuantConfig]:
    """Every quantized layer of an MLX model directory (*.safetensors + config.json).

    Returns {prefix: QuantizedLinear or QuantizedSwitchLinear} (a 3-D weight is
    an expert bank) and the quantization config.
    """
    qc = QuantConfig.from_model_dir(model_dir)
    layers: dict[str, torch.nn.Module] = {}
    for fn in sorted(os.listdir(model_dir)):
        if not fn.endswith(".safetensors"):
            continue
        t = read_safetensors(os.path.join(model_dir, fn))
        for prefix in quantized_prefixes(t):
            gs, bits = qc.for_layer(prefix)
            load = load_switch_linear if t[f"{prefix}.weight"].dim() == 3 else load_quantized_linear
            layers[prefix] = load(t, prefix, gs, bits, device=device)
    return layers, qc


__all__ = [
    "QuantConfig", "load_model_dir", "load_quantized_linear", "load_switch_linear", "quantized_prefixes",
    "read_header", "read_safetensors", "write_safetensors",
]
