// floor.cu -- measurement hook: a plain streaming read of a device buffer.
//
// The benchmark times a chain of these reads with the byte sizes of a decode
// layer's projections, launched exactly like the decode kernel (programmatic
// stream serialization, CUDA graphs).  That chain is the HBM floor a separate
// launch per projection can reach on the machine at hand; the decode kernel's
// time is reported against it.  Nothing on the product path calls this.

#include "common.cuh"
#include "tma.cuh"

namespace qmm {

__global__ void __launch_bounds__(256) stream_read_kernel(const uint4* __restrict__ p, long long n16,
                                                          uint32_t* __restrict__ sink) {
    pdl_launch_dependents();
    pdl_wait();
    uint32_t acc = 0;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x) {
        const uint4 v = ldg_stream_v4(p + i);
        acc ^= v.x ^ v.y ^ v.z ^ v.w;
    }
    // keeps the loads live; the sink only ever receives a value when the xor is exactly this pattern
    if (acc == 0x9E3779B9u) sink[threadIdx.x] = acc;
}

}  // namespace qmm

extern "C" QMM_API int qmm_stream_read(const void* p, size_t bytes, int blocks, void* sink, void* stream) {
    using namespace qmm_host;
    if (!p || !sink || ((uintptr_t)p & 15u) || (bytes & 15u) || blocks < 1 || blocks > 65535) {
        set_error("stream_read: p and sink non-null, p 16-byte aligned, bytes a multiple of 16, 1 <= blocks <= 65535");
        return QMM_EINVAL;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, qmm::stream_read_kernel, static_cast<const uint4*>(p),
                                             (long long)(bytes / 16), static_cast<uint32_t*>(sink));
    if (e != cudaSuccess) cudaGetLastError();
    return cuda_status(e, "stream_read launch");
}
