// torch_ops.cpp -- the public ops as PyTorch custom operators
// (torch.ops.mlxturbo_b200.*) over the C ABI of libmlxturbo_b200.so.
//
// A decode step makes one call per projection, and a projection runs for
// 4-14 us on the device, so the host time of a call bounds the end-to-end
// rate.  Through ctypes a call costs ~10 us (argument conversion, the stream
// handle, the workspace look-up, Python-side checks).  These operators do the
// same work in C++ behind the PyTorch dispatcher: the checks, the tensors'
// device pointers, the current CUDA stream, and one zeroed device workspace
// per device kept here (sized on demand; the decode kernels leave its counter
// block zero and tag their partial sums with a per-call epoch, exactly as with
// the Python layer's workspace).
//
// Signatures follow mx.quantized_matmul (mlxturbo/kernels/dispatch.py:317-327)
// with transpose=True, mode="affine"; an `out` tensor of the result shape may
// be given to reuse the output buffer.  Argument errors raise ValueError (a
// CPU tensor among the arguments included), unsupported dtypes / shapes
// NotImplementedError, with the library's message.  ops.quantized_matmul
// calls these directly and leaves every check to them.

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>
#include <torch/types.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <unordered_map>

#include "../../include/mlxturbo_b200.h"

namespace {

// Error messages are formatted here with vsnprintf and handed to the check
// macros as one string: a message built by the macros' own stream formatting
// from several arguments (numbers, sizes) crashed the process (SIGSEGV) in
// this extension build, while a single string argument raises cleanly.
enum class Err { kValue, kNotImplemented, kRuntime };

[[noreturn]] void fail(Err kind, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    const char* m = buf;
    if (kind == Err::kValue) TORCH_CHECK_VALUE(false, m);
    if (kind == Err::kNotImplemented) TORCH_CHECK_NOT_IMPLEMENTED(false, m);
    TORCH_CHECK(false, m);
    __builtin_unreachable();
}

std::string dims(at::IntArrayRef d) {
    std::string r = "(";
    for (size_t i = 0; i < d.size(); ++i) {
        char b[32];
        std::snprintf(b, sizeof b, i ? ", %lld" : "%lld", (long long)d[i]);
        r += b;
    }
    return r + ")";
}

int dtype_code(const at::Tensor& x) {
    if (x.scalar_type() == at::kBFloat16) return QMM_BF16;
    if (x.scalar_type() == at::kHalf) return QMM_F16;
    fail(Err::kNotImplemented, "activations must be bfloat16 or float16, got %s", c10::toString(x.scalar_type()));
}

void check(int rc, const char* what) {
    if (rc == QMM_OK) return;
    const Err kind = rc == QMM_EUNSUPPORTED ? Err::kNotImplemented : rc == QMM_EINVAL ? Err::kValue : Err::kRuntime;
    fail(kind, "%s: %s: %s", what, qmm_status_string(rc), qmm_last_error());
}

// A zeroed uint8 buffer of at least `bytes` on `device`, kept for the process.
// Growing it replaces the buffer (the old one is released in stream order by
// the caching allocator); a new buffer starts at zero, as the kernels need.
at::Tensor& decode_workspace(const at::Device& device, size_t bytes) {
    static std::mutex mu;
    static std::unordered_map<int, at::Tensor> bufs;
    std::lock_guard<std::mutex> lock(mu);
    at::Tensor& buf = bufs[device.index()];
    if (!buf.defined() || (size_t)buf.numel() < bytes) {
        size_t size = 1u << 20;
        while (size < bytes) size <<= 1;
        buf = at::zeros({(int64_t)size}, at::TensorOptions().dtype(at::kByte).device(device));
    }
    return buf;
}

at::Tensor contiguous16(const at::Tensor& t) {
    at::Tensor c = t.contiguous();
    if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16) c = c.clone();
    return c;
}

at::Tensor run_quantized_matmul(const at::Tensor& x_in, const at::Tensor& w_in, const at::Tensor& scales_in,
                                const at::Tensor& biases_in, int64_t group_size, int64_t bits,
                                const at::Tensor* out) {
    if (!(x_in.is_cuda() && w_in.is_cuda() && scales_in.is_cuda() && biases_in.is_cuda()))
        fail(Err::kValue, "mlxturbo_b200 ops take CUDA tensors (there is no CPU path)");
    if (!(w_in.device() == x_in.device() && scales_in.device() == x_in.device() &&
          biases_in.device() == x_in.device() && (!out || out->device() == x_in.device())))
        fail(Err::kValue, "x, w, scales, biases and out must be on one device");
    if (x_in.dim() < 1) fail(Err::kValue, "x must have at least one dimension");
    const int dt = dtype_code(x_in);
    const at::Tensor x = contiguous16(x_in), w = contiguous16(w_in);
    const at::Tensor s = scales_in.contiguous(), b = biases_in.contiguous();
    if (s.scalar_type() != x.scalar_type() || b.scalar_type() != x.scalar_type())
        fail(Err::kValue, "scales and biases must have the activations' dtype");
    const int64_t K = x.size(-1), N = w.dim() == 2 ? w.size(0) : -1, M = K ? x.numel() / K : 0;
    if (!(w.dim() == 2 && w.size(1) * 32 == K * bits))
        fail(Err::kValue, "w shape %s does not match K=%lld bits=%lld", dims(w.sizes()).c_str(), (long long)K,
             (long long)bits);
    if (!(group_size > 0 && K % group_size == 0 && s.dim() == 2 && s.size(0) == N && s.size(1) == K / group_size &&
          b.sizes() == s.sizes()))
        fail(Err::kValue, "scales/biases shape %s != (%lld, %lld)", dims(s.sizes()).c_str(), (long long)N,
             (long long)(K / (group_size > 0 ? group_size : 1)));
    c10::cuda::CUDAGuard guard(x.device());
    std::vector<int64_t> shape(x.sizes().begin(), x.sizes().end());
    shape.back() = N;
    at::Tensor y;
    if (out) {
        y = *out;
        if (!(y.is_contiguous() && y.sizes() == at::IntArrayRef(shape) && y.scalar_type() == x.scalar_type() &&
              reinterpret_cast<uintptr_t>(y.data_ptr()) % 16 == 0))
            fail(Err::kValue, "out must be a contiguous, 16-byte aligned tensor of the result shape %s and x's dtype",
                 dims(at::IntArrayRef(shape)).c_str());
    } else {
        y = at::empty(shape, x.options());
    }
    if (M == 0) return y;
    const size_t need = qmm_quantized_matmul_workspace_size(M, N, K, (int)group_size, (int)bits);
    void* ws = nullptr;
    size_t ws_bytes = 0;
    if (need) {
        at::Tensor& buf = decode_workspace(x.device(), need);
        ws = buf.data_ptr();
        ws_bytes = (size_t)buf.numel();
    }
    const cudaStream_t st = at::cuda::getCurrentCUDAStream(x.device().index()).stream();
    check(qmm_quantized_matmul(x.data_ptr(), static_cast<const uint32_t*>(w.data_ptr()), s.data_ptr(), b.data_ptr(),
                               y.data_ptr(), M, N, K, (int)group_size, (int)bits, dt, ws, ws_bytes, st),
          "quantized_matmul");
    return y;
}

at::Tensor quantized_matmul(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scales,
                            const at::Tensor& biases, int64_t group_size, int64_t bits) {
    return run_quantized_matmul(x, w, scales, biases, group_size, bits, nullptr);
}

at::Tensor& quantized_matmul_out(const at::Tensor& x, const at::Tensor& w, const at::Tensor& scales,
                                 const at::Tensor& biases, int64_t group_size, int64_t bits, at::Tensor& out) {
    run_quantized_matmul(x, w, scales, biases, group_size, bits, &out);
    return out;
}

// All-CPU arguments: the same error as a CPU tensor among CUDA ones.
at::Tensor quantized_matmul_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&, int64_t,
                                int64_t) {
    fail(Err::kValue, "mlxturbo_b200 ops take CUDA tensors (there is no CPU path)");
}

at::Tensor& quantized_matmul_out_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                     int64_t, int64_t, at::Tensor& out) {
    fail(Err::kValue, "mlxturbo_b200 ops take CUDA tensors (there is no CPU path)");
}

}  // namespace

TORCH_LIBRARY(mlxturbo_b200, m) {
    m.def("quantized_matmul(Tensor x, Tensor w, Tensor scales, Tensor biases, int group_size=64, int bits=4) "
          "-> Tensor");
    m.def("quantized_matmul_out(Tensor x, Tensor w, Tensor scales, Tensor biases, int group_size, int bits, "
          "*, Tensor(a!) out) -> Tensor(a!)");
}

TORCH_LIBRARY_IMPL(mlxturbo_b200, CUDA, m) {
    m.impl("quantized_matmul", &quantized_matmul);
    m.impl("quantized_matmul_out", &quantized_matmul_out);
}

TORCH_LIBRARY_IMPL(mlxturbo_b200, CPU, m) {
    m.impl("quantized_matmul", &quantized_matmul_cpu);
    m.impl("quantized_matmul_out", &quantized_matmul_out_cpu);
}
