// layout.cu -- MLX affine quantisation on the device (weight conversion).
//
// Restates MLX 0.32.2 affine_quantize as used through mx.quantize by the
// reference's converters (mlxturbo/rebit.py:103-121): per group the min/max,
// a scale nudged so that 0.0 lands on the grid, codes rint((w - b)/s) clipped
// to [0, 2^bits - 1], scales/biases rounded to T afterwards.  One thread per
// (row, group); a group always fills whole 32-bit words of the packed row
// (group_size * bits is a multiple of 32), so threads never share a word.

#include "common.cuh"

namespace qmm {

template <bool F16>
__global__ void quantize_kernel(const float* __restrict__ w, uint32_t* __restrict__ wq, uint16_t* __restrict__ sc,
                                uint16_t* __restrict__ bi, long long N, int K, int gs, int bits) {
    using H = Half<F16>;
    const int G = K / gs;
    const long long total = N * (long long)G;
    const float n_bins = (float)((1 << bits) - 1);
    const long long wrow = (long long)K * bits / 32;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long n = idx / G;
        const int g = (int)(idx - n * G);
        const float* v = w + n * K + (long long)g * gs;
        float mx = v[0], mn = v[0];
        for (int i = 1; i < gs; ++i) {
            mx = fmaxf(mx, v[i]);
            mn = fminf(mn, v[i]);
        }
        const bool mask = fabsf(mn) > fabsf(mx);
        float scale = __fdiv_rn(__fsub_rn(mx, mn), n_bins);
        if (scale < 1e-7f) scale = 1e-7f;
        if (!mask) scale = -scale;
        const float edge = mask ? mn : mx;
        const float q0 = rintf(__fdiv_rn(edge, scale));
        float bias = 0.0f;
        if (q0 != 0.0f) {
            scale = __fdiv_rn(edge, q0);
            bias = edge;
        }
        uint32_t* out = wq + n * wrow + (long long)g * gs * bits / 32;
        unsigned long long acc = 0;
        int nbits = 0, wi = 0;
        for (int i = 0; i < gs; ++i) {
            float q = rintf(__fdiv_rn(__fsub_rn(v[i], bias), scale));
            q = fminf(fmaxf(q, 0.0f), n_bins);
            acc |= (unsigned long long)(uint32_t)q << nbits;
            nbits += bits;
            if (nbits >= 32) {
                out[wi++] = (uint32_t)acc;
                acc >>= 32;
                nbits -= 32;
            }
        }
        sc[idx] = H::from_f32(scale);
        bi[idx] = H::from_f32(bias);
    }
}

}  // namespace qmm

namespace qmm_host {

int launch_quantize(const float* w, uint32_t* wq, uint16_t* sc, uint16_t* bi, long long N, int K, int gs, int bits,
                    bool f16, cudaStream_t st) {
    const long long total = N * (K / gs);
    if (total == 0) return QMM_OK;
    long long blocks = (total + 127) / 128;
    if (blocks > 148 * 64) blocks = 148 * 64;
    if (f16) qmm::quantize_kernel<true><<<(unsigned)blocks, 128, 0, st>>>(w, wq, sc, bi, N, K, gs, bits);
    else qmm::quantize_kernel<false><<<(unsigned)blocks, 128, 0, st>>>(w, wq, sc, bi, N, K, gs, bits);
    return cuda_status(cudaGetLastError(), "quantize launch");
}

}  // namespace qmm_host
