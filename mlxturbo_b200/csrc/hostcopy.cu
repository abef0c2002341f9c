// hostcopy.cu -- small host <-> device transfers as one kernel.
//
// A decode step moves a few hundred KB between pinned host memory and the
// device (the step's activations in, its outputs back).  A copy-engine
// transfer of that size costs several microseconds of setup per direction on
// the step's critical path; a kernel that reads (or writes) the pinned pages
// directly over the host link starts like any other launch.  Pinned memory
// is device-addressable under unified virtual addressing, which the entry
// point checks for both pointers before it launches.
//
// Host memory is read with ld.global.cv (no cached copy is reused: the host
// may have rewritten the buffer since the last call) and written with
// st.global.wt (written through to system memory), so a reader on the host
// sees the data once the stream has been synchronised.

#include "common.cuh"

namespace qmm {

__global__ void __launch_bounds__(256) copy16_kernel(const uint4* src, uint4* dst, long long n16) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n16; i += (long long)gridDim.x * blockDim.x) {
        uint4 v;
        asm volatile("ld.global.cv.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(src + i));
        asm volatile("st.global.wt.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(dst + i), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
    }
}

}  // namespace qmm

namespace {

// Whether the device can address p as it is (device memory, managed memory,
// or pinned host memory mapped at the same address).
bool device_addressable(const void* p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) return true;
    return at.type == cudaMemoryTypeHost && at.devicePointer == p;
}

}  // namespace

extern "C" QMM_API int qmm_copy_kernel(void* dst, const void* src, size_t bytes, void* stream) {
    using namespace qmm_host;
    if (bytes == 0) return QMM_OK;
    if (!dst || !src || (((uintptr_t)dst | (uintptr_t)src) & 15u) || (bytes & 15u)) {
        set_error("copy_kernel: dst and src non-null and 16-byte aligned, bytes a multiple of 16");
        return QMM_EINVAL;
    }
    if (!device_addressable(dst) || !device_addressable(src)) {
        set_error("copy_kernel: dst or src is not device-addressable (pageable host memory): use cudaMemcpyAsync");
        return QMM_EINVAL;
    }
    const long long n16 = (long long)(bytes / 16);
    long long blocks = (n16 + 255) / 256;
    if (blocks > 148 * 4) blocks = 148 * 4;
    qmm::copy16_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), static_cast<uint4*>(dst), n16);
    return cuda_status(cudaGetLastError(), "copy_kernel launch");
}
