// argmax.cu -- greedy sampling over stored logits: per row, the largest
// (logit, index) key, for the lm_head shapes the fused integer-MMA epilogue
// does not cover (M > 8, or matrices below its size rule).
//
// Key of a (logit, index) pair: (order-preserving bits of the f32 logit) << 32
// | (0xFFFFFFFF - index), so the maximum key is the largest logit and, among
// equal logits, the smallest index (a single-device argmax's first
// occurrence).  The same key as the integer-MMA kernel's fused epilogue, so a
// sharded lm_head can combine ranks' keys with one max.
// (Caller: mlxturbo/spec.py:388-408 SpecEngine._head takes the argmax of the
// verify logits.)

#include "common.cuh"

namespace qmm {

QMM_DEVINL unsigned long long argmax_key_host(float f, long long n) {
    const uint32_t u = f == 0.0f ? 0u : __float_as_uint(f);  // -0 ties with +0, as in argmax
    const uint32_t mono = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)mono << 32) | (0xFFFFFFFFu - (uint32_t)n);
}

// One thread per 8 consecutive logits of a row (16-byte load), a warp max,
// one atomicMax per warp.  keys must start at zero.
template <bool F16>
__global__ void row_argmax_kernel(const uint16_t* y, int M, int N, long long n_offset, unsigned long long* keys) {
    using H = Half<F16>;
    const int m = blockIdx.y;
    const long long c8 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long n0 = c8 * 8;
    unsigned long long key = 0ull;
    if (n0 < N) {
        const uint16_t* p = y + (long long)m * N + n0;
        if (n0 + 8 <= N && ((reinterpret_cast<uintptr_t>(p) & 15u) == 0)) {
            const uint4 v = ld_v4(p);  // y: the previous kernel's output
            const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const unsigned long long k0 = argmax_key_host(H::lo_f32(u[j]), n_offset + n0 + 2 * j);
                const unsigned long long k1 = argmax_key_host(H::hi_f32(u[j]), n_offset + n0 + 2 * j + 1);
                key = k0 > key ? k0 : key;
                key = k1 > key ? k1 : key;
            }
        } else {
            for (long long n = n0; n < N && n < n0 + 8; ++n) {
                const unsigned long long k = argmax_key_host(H::to_f32(ld_dep(p + (n - n0))), n_offset + n);
                key = k > key ? k : key;
            }
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
        key = k2 > key ? k2 : key;
    }
    if ((threadIdx.x & 31) == 0 && key) atomicMax(keys + m, key);
}

}  // namespace qmm

namespace qmm_host {

int launch_row_argmax(const uint16_t* y, int M, int N, long long n_offset, unsigned long long* keys, bool f16,
                      cudaStream_t st) {
    const long long c8 = ((long long)N + 7) / 8;
    dim3 grid((unsigned)((c8 + 255) / 256), (unsigned)M);
    if (f16) qmm::row_argmax_kernel<true><<<grid, 256, 0, st>>>(y, M, N, n_offset, keys);
    else qmm::row_argmax_kernel<false><<<grid, 256, 0, st>>>(y, M, N, n_offset, keys);
    return cuda_status(cudaGetLastError(), "row_argmax launch");
}

}  // namespace qmm_host
