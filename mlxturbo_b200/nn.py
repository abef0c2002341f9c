"""torch modules over the quantized ops: the layer types the reference's
callers hold (mlx.nn.QuantizedLinear and mlx-lm's QuantizedSwitchLinear /
SwitchGLU), with MLX's parameter names (weight, scales, biases, bias) and
call semantics, so model code ported from MLX keeps its shape contracts."""

from __future__ import annotations

import torch
from torch import nn

from . import ops


class QuantizedLinear(nn.Module):
    """y = x @ dequant(weight)^T (+ bias); weight uint32-as-int32 [N, K*bits/32]."""

    def __init__(self, input_dims: int, output_dims: int, bias: bool = False, group_size: int = 64, bits: int = 4,
                 mode: str = "affine", dtype=torch.bfloat16, device=None):
        super().__init__()
        self.group_size, self.bits, self.mode = group_size, bits, mode
        self.input_dims, self.output_dims = input_dims, output_dims
        self.register_buffer("weight", torch.zeros((output_dims, input_dims * bits // 32), dtype=torch.int32,
                                                   device=device))
        self.register_buffer("scales", torch.zeros((output_dims, input_dims // group_size), dtype=dtype,
                                                   device=device))
        self.register_buffer("biases", torch.zeros_like(self.scales))
        self.bias = nn.Parameter(torch.zeros(output_dims, dtype=dtype, device=device)) if bias else None

    @classmethod
    def from_float(cls, w: torch.Tensor, bias: torch.Tensor | None = None, group_size: int = 64, bits: int = 4,
                   dtype=torch.bfloat16):
        """Quantise a float weight [N, K] (mx.quantize, affine) into a new layer."""
        N, K = w.shape
        layer = cls(K, N, bias is not None, group_size, bits, dtype=dtype, device=w.device)
        wq, s, b = ops.quantize(w, group_size, bits, dtype=dtype)
        layer.weight.copy_(wq)
        layer.scales.copy_(s)
        layer.biases.copy_(b)
        if bias is not None:
            layer.bias.data.copy_(bias.to(dtype))
        return layer

    def forward(self, x):
        y = ops.quantized_matmul(x, self.weight, self.scales, self.biases, group_size=self.group_size,
                                 bits=self.bits, mode=self.mode)
        return y if self.bias is None else y + self.bias


class QuantizedSwitchLinear(nn.Module):
    """Expert bank: weight [E, N, K*bits/32]; forward(x, indices, sorted_indices)."""

    def __init__(self, input_dims: int, output_dims: int, num_experts: int, bias: bool = False,
                 group_size: int = 64, bits: int = 4, mode: str = "affine", dtype=torch.bfloat16, device=None):
        super().__init__()
        self.group_size, self.bits, self.mode = group_size, bits, mode
        self.register_buffer("weight", torch.zeros((num_experts, output_dims, input_dims * bits // 32),
                                                   dtype=torch.int32, device=device))
        self.register_buffer("scales", torch.zeros((num_experts, output_dims, input_dims // group_size),
                                                   dtype=dtype, device=device))
        self.register_buffer("biases", torch.zeros_like(self.scales))
        self.bias = nn.Parameter(torch.zeros(num_experts, output_dims, dtype=dtype, device=device)) if bias else None

    @property
    def num_experts(self) -> int:
        return self.weight.shape[0]

    def slice_experts(self, start: int, stop: int) -> "QuantizedSwitchLinear":
        """A new layer holding experts [start, stop) of this one (expert parallelism)."""
        E, N, kw = self.weight.shape
        out = QuantizedSwitchLinear(kw * 32 // self.bits, N, stop - start, self.bias is not None, self.group_size,
                                    self.bits, self.mode, dtype=self.scales.dtype, device=self.weight.device)
        out.weight.copy_(self.weight[start:stop])
        out.scales.copy_(self.scales[start:stop])
        out.biases.copy_(self.biases[start:stop])
        if self.bias is not None:
            out.bias.data.copy_(self.bias[start:stop])
        return out

    def forward(self, x, indices, sorted_indices: bool = False):
        """x (..., 1, K) or (rows, 1, K), indices (...) -> (..., 1, N) like mx.gather_qmm."""
        y = ops.gather_qmm(x, self.weight, self.scales, self.biases, rhs_indices=indices, transpose=True,
                           group_size=self.group_size, bits=self.bits, mode=self.mode,
                           sorted_indices=sorted_indices)
        if self.bias is not None:
            y = y + self.bias[indices].unsqueeze(-2)
        return y


def swiglu(x_up: torch.Tensor, x_gate: torch.Tensor) -> torch.Tensor:
    """mlx-lm SwitchGLU activation: silu(gate) * up."""
    return torch.nn.functional.silu(x_gate) * x_up


class SwitchGLU(nn.Module):
    """mlx-lm SwitchGLU over quantized experts (gate/up/down projections)."""

    def __init__(self, input_dims: int, hidden_dims: int, num_experts: int, group_size: int = 64, bits: int = 4,
                 dtype=torch.bfloat16, device=None):
        super().__init__()
        self.gate_proj = QuantizedSwitchLinear(input_dims, hidden_dims, num_experts, False, group_size, bits,
                                               dtype=dtype, device=device)
        self.up_proj = QuantizedSwitchLinear(input_dims, hidden_dims, num_experts, False, group_size, bits,
                                             dtype=dtype, device=device)
        self.down_proj = QuantizedSwitchLinear(hidden_dims, input_dims, num_experts, False, group_size, bits,
                                               dtype=dtype, device=device)
        self.activation = swiglu
        self._fused = None

    def fused_gate_up(self):
        """The gate and up banks as one [E, 2I, ...] bank, rows interleaved per
        16-row block (gate rows 8b..8b+7, then up rows 8b..8b+7), for the
        gathered matmul's SwiGLU epilogue.  Built once on the device and cached;
        call ``refresh_fused()`` after changing the weights in place."""
        if self._fused is None:
            g, u = self.gate_proj, self.up_proj
            E, I = g.weight.shape[0], g.weight.shape[1]
            if I % 8 or u.weight.shape != g.weight.shape or g.group_size != u.group_size or g.bits != u.bits:
                raise NotImplementedError("fused gate/up needs matching banks with intermediate size % 8 == 0")

            def inter(a, b):
                return torch.stack([a.reshape(E, I // 8, 8, -1), b.reshape(E, I // 8, 8, -1)], dim=2).reshape(
                    E, 2 * I, -1).contiguous()

            self._fused = (inter(g.weight, u.weight), inter(g.scales, u.scales), inter(g.biases, u.biases))
        return self._fused

    def refresh_fused(self):
        self._fused = None

    def slice_experts(self, start: int, stop: int) -> "SwitchGLU":
        """A new SwitchGLU holding experts [start, stop) of all three projections."""
        out = SwitchGLU.__new__(SwitchGLU)
        nn.Module.__init__(out)
        out.gate_proj = self.gate_proj.slice_experts(start, stop)
        out.up_proj = self.up_proj.slice_experts(start, stop)
        out.down_proj = self.down_proj.slice_experts(start, stop)
        out.activation = self.activation
        out._fused = None
        return out

    def forward(self, x, indices):
        """x (..., K), indices (..., top_k) -> (..., top_k, K)."""
        xx = x.unsqueeze(-2).unsqueeze(-3)  # (..., 1, 1, K)
        do_sort = indices.numel() >= 64
        if do_sort:
            flat = indices.reshape(-1)
            order = torch.argsort(flat, stable=True)
            inv = torch.argsort(order)
            top_k = indices.shape[-1]
            xs = xx.reshape(-1, 1, x.shape[-1])[order // top_k]
            idx = flat[order]
        else:
            xs, idx = xx, indices
        up = self.up_proj(xs, idx, sorted_indices=do_sort)
        gate = self.gate_proj(xs, idx, sorted_indices=do_sort)
        out = self.down_proj(self.activation(up, gate), idx, sorted_indices=do_sort)
        if do_sort:
            out = out[inv].reshape(*indices.shape, 1, -1)
        return out.squeeze(-2)
