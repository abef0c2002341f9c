"""PyTorch-facing quantized matmul ops over the C ABI.

These keep MLX's operator signatures so callers written against
``mx.quantized_matmul`` / ``mx.gather_qmm`` (the reference's stock path,
mlxturbo/kernels/dispatch.py:317-327, fused.py:3105-3116) call them unchanged:

    quantized_matmul(x, w, scales, biases, transpose=True, group_size=64, bits=4, mode="affine")
    gather_qmm(x, w, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=64, bits=4, mode="affine", sorted_indices=False)

Tensors live on a CUDA device; weights are uint32 (MLX packing).  torch has no
uint32 arithmetic on CUDA, so int32 tensors holding the same bits are accepted
as well.  Every call goes through libmlxturbo_b200.so on the current stream;
there is no CPU path.
"""

from __future__ import annotations

import math

import torch

from . import _lib

_DTYPE = {torch.bfloat16: _lib.QMM_BF16, torch.float16: _lib.QMM_F16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise NotImplementedError(f"activations must be bfloat16 or float16, got {t.dtype}") from None


# the current stream's handle without building a torch.cuda.Stream object
# (~0.2 us instead of ~2 us per call)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("mlxturbo_b200 ops take CUDA tensors (there is no CPU path)")


def _contig(t: torch.Tensor) -> torch.Tensor:
    if not t.is_contiguous() or (t.data_ptr() % 16):
        t = t.contiguous()
        if t.data_ptr() % 16:
            t = t.clone()
    return t


def _check_mode(mode: str, transpose: bool) -> None:
    if mode != "affine":
        raise NotImplementedError(f"mode={mode!r}: only affine quantisation is implemented")
    if not transpose:
        raise NotImplementedError("transpose=False is not on the hot path (the reference only uses transpose=True)")


# --------------------------------------------------------------------------
# per-device scratch
# --------------------------------------------------------------------------
_WORKSPACE: dict[tuple[int, bool], torch.Tensor] = {}


def workspace(device: torch.device, nbytes: int, zeroed: bool = False) -> torch.Tensor:
    """A cached uint8 scratch buffer of at least nbytes on `device`.

    ``zeroed`` buffers start at zero and the kernels that use them (the decode
    kernel's tile counters) leave them zero after every call.  Stream-ordered
    use only: calls on different streams of one device must not overlap (the
    reference's MLX path is single-stream per model).
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _WORKSPACE.get((idx, zeroed))
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20)
        size = 1 << math.ceil(math.log2(size))
        buf = (torch.zeros if zeroed else torch.empty)(size, dtype=torch.uint8, device=device)
        _WORKSPACE[(idx, zeroed)] = buf
    return buf


# decode workspace bytes per (M, N, K, group_size, bits): a pure function of
# the shape, asked of the library once per shape
_WS_NEED: dict[tuple[int, int, int, int, int], int] = {}


def _decode_workspace(lib, x: torch.Tensor, M: int, N: int, K: int, group_size: int, bits: int):
    key = (M, N, K, group_size, bits)
    need = _WS_NEED.get(key)
    if need is None:
        need = _WS_NEED[key] = int(lib.qmm_quantized_matmul_workspace_size(M, N, K, group_size, bits))
    if not need:
        return None, 0
    buf = _WORKSPACE.get((x.get_device(), True))
    if buf is None or buf.numel() < need:
        buf = workspace(x.device, need, zeroed=True)
    return buf.data_ptr(), buf.numel()


# --------------------------------------------------------------------------
# quantized_matmul
# --------------------------------------------------------------------------
_QMM_OPS: tuple | None = None  # (plain, out) operator overloads; () without the operator library


def _qmm_ops() -> tuple:
    global _QMM_OPS
    tops = _lib.torch_ops()
    _QMM_OPS = (tops.quantized_matmul.default, tops.quantized_matmul_out.default) if tops is not None else ()
    return _QMM_OPS


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4, mode: str = "affine",
                     *, out: torch.Tensor | None = None) -> torch.Tensor:
    """y[..., N] = x[..., K] @ dequant(w)^T (mx.quantized_matmul, transpose=True).

    Runs through the PyTorch operator ``torch.ops.mlxturbo_b200.quantized_matmul``
    (C++: the argument checks, the stream and the workspace in a few
    microseconds of host time) when libmlxturbo_b200_torch.so is built, else
    through the ctypes binding with the same checks in Python; both call the
    same C ABI entry and raise the same exception types.
    """
    if mode != "affine" or not transpose:
        _check_mode(mode, transpose)
    if biases is None:
        raise NotImplementedError("affine mode needs biases")
    fast = _QMM_OPS if _QMM_OPS is not None else _qmm_ops()
    if fast:
        if out is None:
            return fast[0](x, w, scales, biases, group_size, bits)
        return fast[1](x, w, scales, biases, group_size, bits, out=out)
    _check_cuda(x, w, scales, biases)
    if x.dim() < 1:
        raise ValueError("x must have at least one dimension")
    K = x.shape[-1]
    N = w.shape[0]
    if w.dim() != 2 or w.shape[1] * 32 != K * bits:
        raise ValueError(f"w shape {tuple(w.shape)} does not match K={K} bits={bits}")
    if scales.shape != (N, K // group_size) or biases.shape != scales.shape:
        raise ValueError(f"scales/biases shape {tuple(scales.shape)} != ({N}, {K // group_size})")
    dt = _dtype_code(x)
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        raise ValueError("scales and biases must have the dtype of x")
    lead = x.shape[:-1]
    M = math.prod(lead)
    x2 = _contig(x.reshape(M, K)) if x.dim() != 2 else _contig(x)
    w = _contig(w)
    scales = _contig(scales)
    biases = _contig(biases)
    if out is None:
        out = torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    elif out.shape != (*lead, N) or out.dtype != x.dtype or not out.is_contiguous() or out.data_ptr() % 16:
        raise ValueError("out must be a contiguous, 16-byte aligned tensor of the result shape and dtype")
    if x.device != w.device or scales.device != x.device or biases.device != x.device or out.device != x.device:
        raise ValueError("x, w, scales, biases and out must be on one device")
    lib = _lib.load()
    ws_ptr, ws_bytes = _decode_workspace(lib, x, M, N, K, group_size, bits) if 0 < M <= 16 else (None, 0)
    dev = x.get_device()
    stream = _raw_stream(dev) if _raw_stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    rc = lib.qmm_quantized_matmul(x2.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), out.data_ptr(),
                                  M, N, K, group_size, bits, dt, ws_ptr, ws_bytes, stream)
    _lib.check(rc, "quantized_matmul")
    return out


def quantized_matmul_argmax(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                            group_size: int = 64, bits: int = 4, *, index_offset: int = 0,
                            out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Logits and greedy keys in one call (C ABI qmm_quantized_matmul_argmax).

    Returns ``(y, keys)``: y [..., N] as quantized_matmul computes it, and
    keys int64 [M] (M = rows of x) with the uint64 key
    ``(order-preserving f32 bits of the max logit) << 32 | (0xFFFFFFFF - index)``
    of each row, index counted from ``index_offset``.  ``argmax_from_keys``
    turns keys (or the max of several shards' keys) into token ids.
    """
    _check_cuda(x, w, scales, biases)
    K = x.shape[-1]
    N = w.shape[0]
    if w.dim() != 2 or w.shape[1] * 32 != K * bits:
        raise ValueError(f"w shape {tuple(w.shape)} does not match K={K} bits={bits}")
    if scales.shape != (N, K // group_size) or biases.shape != scales.shape:
        raise ValueError(f"scales/biases shape {tuple(scales.shape)} != ({N}, {K // group_size})")
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        raise ValueError("scales and biases must have the dtype of x")
    lead = x.shape[:-1]
    M = math.prod(lead)
    x2 = _contig(x.reshape(M, K))
    w, scales, biases = _contig(w), _contig(scales), _contig(biases)
    if out is None:
        out = torch.empty((*lead, N), dtype=x.dtype, device=x.device)
    keys = torch.empty(M, dtype=torch.int64, device=x.device)
    lib = _lib.load()
    ws_ptr, ws_bytes = _decode_workspace(lib, x, M, N, K, group_size, bits) if 0 < M <= 16 else (None, 0)
    rc = lib.qmm_quantized_matmul_argmax(x2.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                         out.data_ptr(), M, N, K, group_size, bits, _dtype_code(x), index_offset,
                                         keys.data_ptr(), ws_ptr, ws_bytes, _stream(x.device))
    _lib.check(rc, "quantized_matmul_argmax")
    return out, keys


_SIGN64 = -(1 << 63)


def max_keys(keys: torch.Tensor, dim: int = 0) -> torch.Tensor:
    """The largest uint64 key along `dim` of an int64 tensor holding the bits."""
    return (keys ^ _SIGN64).max(dim=dim).values ^ _SIGN64


def argmax_from_keys(keys: torch.Tensor) -> torch.Tensor:
    """Token ids (int64) of greedy keys."""
    return 0xFFFFFFFF - (keys & 0xFFFFFFFF)


def qmv_explicit(x, w, scales, biases, *, group_size=64, bits=4, rows_per_warp=1, k_warps=1):
    """The M<=16 kernel with an explicit tile shape (tests and tuning)."""
    _check_cuda(x, w, scales, biases)
    M, K = x.shape
    N = w.shape[0]
    x, w, scales, biases = (_contig(t) for t in (x, w, scales, biases))
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    rc = _lib.load().qmm_qmv_explicit(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                      out.data_ptr(), M, N, K, group_size, bits, _dtype_code(x), rows_per_warp,
                                      k_warps, _stream(x.device))
    _lib.check(rc, "qmv_explicit")
    return out


def qmv_i8(x, w, scales, biases, *, group_size=64, bits=4, out=None):
    """The integer-MMA decode kernel (M <= 8, C ABI qmm_qmv_i8) called directly;
    raises NotImplementedError for shapes it does not take."""
    _check_cuda(x, w, scales, biases)
    M, K = x.shape
    N = w.shape[0]
    x, w, scales, biases = (_contig(t) for t in (x, w, scales, biases))
    if out is None:
        out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    lib = _lib.load()
    need = int(lib.qmm_quantized_matmul_workspace_size(M, N, K, group_size, bits))
    ws = workspace(x.device, max(need, 1), zeroed=True)
    rc = lib.qmm_qmv_i8(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), out.data_ptr(), M, N, K,
                        group_size, bits, _dtype_code(x), ws.data_ptr(), ws.numel(), _stream(x.device))
    _lib.check(rc, "qmv_i8")
    return out


def prefill_explicit(x, w, scales, biases, *, group_size=64, bits=4, tokens_per_cta=256):
    """The tensor-core prefill kernel for any M with an explicit token tile (tests and tuning)."""
    _check_cuda(x, w, scales, biases)
    M, K = x.shape
    N = w.shape[0]
    x, w, scales, biases = (_contig(t) for t in (x, w, scales, biases))
    out = torch.empty((M, N), dtype=x.dtype, device=x.device)
    rc = _lib.load().qmm_prefill_explicit(x.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                                          out.data_ptr(), M, N, K, group_size, bits, _dtype_code(x), tokens_per_cta,
                                          _stream(x.device))
    _lib.check(rc, "prefill_explicit")
    return out


def device_error(reset: bool = True) -> int:
    """Nonzero if a bounded wait inside a tensor-core kernel gave up (synchronises)."""
    return int(_lib.load().qmm_device_error(int(reset)))


def qmv_k_warps(N: int, K: int, group_size: int = 64) -> int:
    return int(_lib.load().qmm_qmv_k_warps(N, K, group_size))


# --------------------------------------------------------------------------
# gather_qmm
# --------------------------------------------------------------------------

def gather_qmm(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               lhs_indices: torch.Tensor | None = None, rhs_indices: torch.Tensor | None = None,
               transpose: bool = True, group_size: int = 64, bits: int = 4, mode: str = "affine",
               sorted_indices: bool = False) -> torch.Tensor:
    """mx.gather_qmm with transpose=True.

    The reference's form (fused.py:3105-3116, SwitchGLU) is x (rows, 1, K),
    rhs_indices (rows,) and an output (rows, 1, N).  Here, as in MLX, the
    output shape is index_shape + (M, N) where x is (..., M, K) with batch
    dims broadcast against the indices; lhs_indices select x batches.
    """
    _check_mode(mode, transpose)
    if rhs_indices is None:
        raise NotImplementedError("gather_qmm without rhs_indices is quantized_matmul")
    _check_cuda(x, w, scales, biases, rhs_indices)
    if w.dim() != 3:
        raise ValueError("w must be [E, N, K*bits/32]")
    E, N = w.shape[0], w.shape[1]
    K = x.shape[-1]
    if w.shape[2] * 32 != K * bits or scales.shape != (E, N, K // group_size) or biases.shape != scales.shape:
        raise ValueError("w/scales/biases do not match x's K, bits and group_size")
    dt = _dtype_code(x)
    Mx = x.shape[-2] if x.dim() >= 2 else 1
    x_batch = x.reshape(-1, Mx, K)
    B = x_batch.shape[0]
    idx_shape = rhs_indices.shape
    rhs = rhs_indices.reshape(-1)
    n_idx = rhs.numel()
    if lhs_indices is not None:
        if lhs_indices.shape != rhs_indices.shape:
            lb, rb = torch.broadcast_tensors(lhs_indices, rhs_indices)
            idx_shape, lhs, rhs = lb.shape, lb.reshape(-1), rb.reshape(-1)
            n_idx = rhs.numel()
        else:
            lhs = lhs_indices.reshape(-1)
    elif B == n_idx:
        lhs = None  # identity
    elif B == 1:
        lhs = torch.zeros(n_idx, dtype=torch.int32, device=x.device)
    else:
        raise ValueError(f"x batch {B} does not broadcast against {n_idx} indices")
    # One output row per (index, activation row).
    x_rows2 = _contig(x_batch.reshape(B * Mx, K))
    if Mx == 1:
        lhs_rows, rhs_rows = lhs, rhs
    else:
        base = (lhs.long() if lhs is not None else torch.arange(n_idx, device=x.device)) * Mx
        lhs_rows = (base[:, None] + torch.arange(Mx, device=x.device)[None, :]).reshape(-1)
        rhs_rows = rhs[:, None].expand(n_idx, Mx).reshape(-1)
    rows = rhs_rows.numel()
    rhs32 = _contig(rhs_rows.to(torch.int32))
    lhs32 = None if lhs_rows is None else _contig(lhs_rows.to(torch.int32))
    out = torch.empty((rows, N), dtype=x.dtype, device=x.device)
    ws_bytes = int(_lib.load().qmm_gather_workspace_size(rows, E))
    ws = workspace(x.device, ws_bytes, zeroed=True)  # starts with the gather kernel's tile counters
    w_, s_, b_ = _contig(w), _contig(scales), _contig(biases)
    rc = _lib.load().qmm_gather_qmm(x_rows2.data_ptr(), w_.data_ptr(), s_.data_ptr(), b_.data_ptr(),
                                    None if lhs32 is None else lhs32.data_ptr(), rhs32.data_ptr(), out.data_ptr(),
                                    rows, x_rows2.shape[0], E, N, K, group_size, bits, dt, int(bool(sorted_indices)),
                                    ws.data_ptr(), ws.numel(), _stream(x.device))
    _lib.check(rc, "gather_qmm")
    return out.reshape(*idx_shape, Mx, N)


# --------------------------------------------------------------------------
# layout helpers
# --------------------------------------------------------------------------

def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64, bits: int = 4,
               mode: str = "affine") -> torch.Tensor:
    """mx.dequantize: T [N, K] from the packed layout (scales' dtype)."""
    _check_mode(mode, True)
    _check_cuda(w, scales, biases)
    N = w.shape[0]
    K = w.shape[1] * 32 // bits
    out = torch.empty((N, K), dtype=scales.dtype, device=w.device)
    w, scales, biases = _contig(w), _contig(scales), _contig(biases)
    rc = _lib.load().qmm_dequantize(w.data_ptr(), scales.data_ptr(), biases.data_ptr(), out.data_ptr(), N, K,
                                    group_size, bits, _dtype_code(scales), _stream(w.device))
    _lib.check(rc, "dequantize")
    return out


def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, mode: str = "affine",
             dtype: torch.dtype | None = None):
    """mx.quantize (affine): (w_q uint32-bits-in-int32 [N, K*bits/32], scales, biases).

    Scales and biases take `dtype` (default: w's dtype if 16-bit, else bf16).
    """
    _check_mode(mode, True)
    _check_cuda(w)
    if w.dim() != 2:
        raise ValueError("quantize takes a 2-D weight")
    N, K = w.shape
    if dtype is None:
        dtype = w.dtype if w.dtype in _DTYPE else torch.bfloat16
    wf = _contig(w.float())
    wq = torch.empty((N, K * bits // 32), dtype=torch.int32, device=w.device)
    sc = torch.empty((N, K // group_size), dtype=dtype, device=w.device)
    bi = torch.empty_like(sc)
    rc = _lib.load().qmm_quantize(wf.data_ptr(), wq.data_ptr(), sc.data_ptr(), bi.data_ptr(), N, K, group_size,
                                  bits, _DTYPE[dtype], _stream(w.device))
    _lib.check(rc, "quantize")
    return wq, sc, bi


def copy_(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """dst <- src with one kernel on the current stream of the CUDA side
    (qmm_copy_kernel), where one side is pinned host memory and the other a
    CUDA tensor: a decode step's activations in and outputs out without a
    copy-engine transfer.  Both contiguous, same dtype and element count,
    16-byte aligned, a multiple of 16 bytes.  Raises ValueError otherwise
    (pageable host memory included: use ``Tensor.copy_``)."""
    if dst.dtype != src.dtype or dst.numel() != src.numel():
        raise ValueError(f"copy_: dst {dst.dtype}[{dst.numel()}] and src {src.dtype}[{src.numel()}] differ")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("copy_: dst and src must be contiguous")
    if not (dst.is_cuda or src.is_cuda):
        raise ValueError("copy_: one side must be a CUDA tensor")
    dev = dst.device if dst.is_cuda else src.device
    nbytes = dst.numel() * dst.element_size()
    _lib.check(_lib.load().qmm_copy_kernel(dst.data_ptr(), src.data_ptr(), nbytes, _stream(dev)), "copy_")
    return dst
