// qmv.cu -- decode / speculative-verify quantized matmul for M <= 16 rows
// (and its expert-gathered form), sm_100a.
//
// Replaces the reference's M=1..16 kernels: MLX qmv_fast (restated in
// mlxturbo/kernels/qmv_small_m.py:79-218), qmv_wide_nocap
// (qmv_wide_nocap.py:77-183), fast_qmm's 8x8 MMA split-K kernel
// (fast_qmm.py:59-139, 158-238) and the expert-segmented gather
// (moe_verify_gather.py:213-876, stock gather_qmv).
//
// Design (B200): the op is HBM bound (0.5625 B per 4-bit weight), so the
// weights are streamed exactly once with coalesced read-once loads and every
// arithmetic step happens in registers:
//   * one warp owns 16*RW weight rows (RW m16 tiles) over a K slice; the CTA's
//     warps split K (fixed group ranges) and reduce through shared memory in
//     warp order -- deterministic, and independent of M;
//   * codes become exact bf16/fp16 integers with one LOP3 per pair
//     ((w >> 4i) & 0x000F000F) | magic, i.e. (offset + q) with offset 128
//     (bf16) or 1024 (fp16);
//   * warp-level tensor-core MMA (m16n8k16) multiplies the code tile by the
//     activations (n = activation rows, up to 8 per MMA, two MMAs for M<=16);
//   * per quantisation group, the MLX qmv factorisation
//     y += s * sum(q*x) + b * sum(x) is applied in fp32, with sum(x) taken by
//     a ones-row MMA on the same tensor pipe and the code offset folded into
//     the bias term: y += s * sum((off+q)*x) + (b - off*s) * sum(x).
// Exact products and fp32 accumulation keep the result within bf16 output
// rounding of the fp32 dequantise-then-matmul reference.
//
// Operand order inside one k16 MMA step is a free permutation of K as long as
// A and B agree; the permutation used here pairs nibble i with nibble i+4 of a
// word (what one LOP3 produces) and PRMT applies the same pairing to x.

#include <stdio.h>

#include "common.cuh"
#include "qmv_args.cuh"

namespace qmm {

// The K loop walks "chunks" of CH = min(group_size, 64) values; a 128-wide
// quantisation group is two chunks sharing one scale and bias.
template <int BITS, int GS>
struct QGeom {
    static constexpr int CH = GS < 64 ? GS : 64;  // K values per chunk
    static constexpr int WPG = CH * BITS / 32;    // packed words per chunk per row
    static constexpr int WPT = WPG / 4;           // words per thread per chunk per row
    static constexpr int VPT = CH / 4;            // values per thread per chunk
    static constexpr int XR = VPT / 2;            // x registers (2 values each) per thread per chunk
    static constexpr int STEPS = CH / 16;         // k16 MMA steps per chunk
    static constexpr int CPG = GS / CH;           // chunks per quantisation group
    static_assert(WPT >= 1 && WPT <= 4, "unsupported bits/group_size");
};

template <int WPT>
QMM_DEVINL void load_words(uint32_t (&dst)[WPT], const uint32_t* p) {
    if constexpr (WPT == 1) {
        dst[0] = ldg_stream_u32(p);
    } else if constexpr (WPT == 2) {
        uint2 v = ldg_stream_v2(p);
        dst[0] = v.x;
        dst[1] = v.y;
    } else {
#pragma unroll
        for (int i = 0; i < WPT; i += 4) {
            uint4 v = ldg_stream_v4(p + i);
            dst[i] = v.x;
            dst[i + 1] = v.y;
            dst[i + 2] = v.z;
            dst[i + 3] = v.w;
        }
    }
}

template <int XR>
QMM_DEVINL void load_x(uint32_t (&dst)[XR], const uint16_t* p, bool valid) {
#pragma unroll
    for (int i = 0; i < XR; i += 4) {
        uint4 v = valid ? ldg_v4(p + 2 * i) : make_uint4(0, 0, 0, 0);
        dst[i] = v.x;
        dst[i + 1] = v.y;
        dst[i + 2] = v.z;
        dst[i + 3] = v.w;
    }
}

// B fragment (b0, b1) of MMA step j from the thread's x registers.
template <int BITS, int XR>
QMM_DEVINL void x_frag(const uint32_t (&xr)[XR], int j, uint32_t& b0, uint32_t& b1) {
    if constexpr (BITS == 4) {
        const int q = j >> 1;
        const uint32_t ra = (j & 1) ? xr[4 * q + 1] : xr[4 * q];
        const uint32_t rb = (j & 1) ? xr[4 * q + 3] : xr[4 * q + 2];
        b0 = prmt(ra, rb, 0x5410);
        b1 = prmt(ra, rb, 0x7632);
    } else {
        const uint32_t ra = xr[2 * j], rb = xr[2 * j + 1];
        b0 = prmt(ra, rb, 0x5410);
        b1 = prmt(ra, rb, 0x7632);
    }
}

template <int BITS, int GS, bool F16, int MT, int RW, int PD, bool GATHER>
__global__ void __launch_bounds__(512) qmv_kernel(QmvArgs args) {
    using G_ = QGeom<BITS, GS>;
    using H = Half<F16>;
    constexpr int WPT = G_::WPT, WPG = G_::WPG, XR = G_::XR, STEPS = G_::STEPS, VPT = G_::VPT;
    constexpr int CH = G_::CH, CPG = G_::CPG;
    constexpr uint32_t MAGIC = H::kMagic;
    constexpr uint32_t MASK = 0x000F000Fu;
    // sum(q*x) = acc - OFF_TOTAL * sum(x) with the code offsets folded.
    constexpr float OFF = H::kOffset;
    constexpr float OFF_TOTAL = BITS == 4 ? OFF : 17.0f * OFF;

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int N = args.N, K = args.K;
    const int G = K / GS;      // scale/bias groups per row
    const int C = K / CH;      // chunks per row

    // ---- rows of activations handled by this CTA ------------------------
    int m_count = args.M;
    int r0 = 0;
    const uint32_t* w = args.w;
    const uint16_t* sc = args.sc;
    const uint16_t* bi = args.bi;
    if constexpr (GATHER) {
        const Segments& sg = args.seg;
        const int item = blockIdx.y;
        const int total = __ldg(sg.tile_prefix + sg.E);
        if (item >= total) return;
        // expert e with tile_prefix[e] <= item < tile_prefix[e+1]
        int lo = 0, hi = sg.E;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (__ldg(sg.tile_prefix + mid) <= item) lo = mid; else hi = mid;
        }
        const int e = lo;
        const int chunk = item - __ldg(sg.tile_prefix + e);
        r0 = __ldg(sg.row_start + e) + 16 * chunk;
        m_count = min(16, __ldg(sg.row_start + e + 1) - r0);
        w += (long long)e * sg.w_stride;
        sc += (long long)e * sg.s_stride;
        bi += (long long)e * sg.s_stride;
    }

    // ---- this warp's chunks ---------------------------------------------
    const int gbase = C / nwarps, grem = C % nwarps;
    const int g0 = warp * gbase + min(warp, grem);
    const int ng = gbase + (warp < grem ? 1 : 0);

    const int n_block = blockIdx.x * (16 * RW);
    const long long wrow = (long long)K * BITS / 32;

    const uint32_t* wp[RW][2];
    const uint16_t* sp[RW][2];
    const uint16_t* bp[RW][2];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int n = n_block + 16 * r + g + 8 * h;
            n = n < N ? n : N - 1;  // rows past N load a valid row; their results are dropped
            wp[r][h] = w + (long long)n * wrow + (long long)g0 * WPG + t * WPT;
            sp[r][h] = sc + (long long)n * G;
            bp[r][h] = bi + (long long)n * G;
        }

    const uint16_t* xp[MT];
    bool xv[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = 8 * mt + g;
        xv[mt] = m < m_count;
        long long src = xv[mt] ? (long long)(r0 + m) : (long long)r0;
        if constexpr (GATHER) {
            if (args.seg.row_src != nullptr && xv[mt]) src = __ldg(args.seg.row_src + r0 + m);
            if (src < 0 || src >= args.seg.x_rows) {  // out-of-range index: contribute zeros, read nothing
                xv[mt] = false;
                src = 0;
            }
        }
        xp[mt] = args.x + src * K + (long long)g0 * CH + t * VPT;
    }

    float res[RW][MT][4];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) res[r][mt][c] = 0.0f;

    const uint32_t ones[4] = {H::kOne2, H::kOne2, H::kOne2, H::kOne2};
    const float zero4[4] = {0.0f, 0.0f, 0.0f, 0.0f};

    // ---- register ring of PD groups of packed words ------------------------
    uint32_t wbuf[PD][RW][2][WPT];
#pragma unroll
    for (int s = 0; s < PD - 1; ++s)
        if (s < ng) {
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int h = 0; h < 2; ++h) load_words<WPT>(wbuf[s][r][h], wp[r][h] + s * WPG);
        }

    for (int i0 = 0; i0 < ng; i0 += PD) {
#pragma unroll
        for (int s = 0; s < PD; ++s) {
            const int i = i0 + s;
            if (i + PD - 1 < ng) {
                const int st = (s + PD - 1) % PD;
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
                        load_words<WPT>(wbuf[st][r][h], wp[r][h] + (long long)(i + PD - 1) * WPG);
            }
            if (i < ng) {
                // activations of this group (L1/L2 resident, shared by all warps)
                uint32_t xr[MT][XR];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) load_x<XR>(xr[mt], xp[mt] + (long long)i * CH, xv[mt]);
                // scale and bias of the chunk's group
                const int grp = (g0 + i) / CPG;
                float s_[RW][2], b_[RW][2];
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        s_[r][h] = H::to_f32(ldg_u16(sp[r][h] + grp));
                        b_[r][h] = H::to_f32(ldg_u16(bp[r][h] + grp));
                    }
                // B fragments and sum(x) of the group
                uint32_t bf[MT][STEPS][2];
                float xs[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
                    for (int j = 0; j < STEPS; ++j) x_frag<BITS, XR>(xr[mt], j, bf[mt][j][0], bf[mt][j][1]);
                    mma16816<F16>(xs[mt], ones, bf[mt][0][0], bf[mt][0][1], zero4);
#pragma unroll
                    for (int j = 1; j < STEPS; ++j) mma16816<F16>(xs[mt], ones, bf[mt][j][0], bf[mt][j][1], xs[mt]);
                }
#pragma unroll
                for (int r = 0; r < RW; ++r) {
                    const uint32_t(&w0)[WPT] = wbuf[s][r][0];
                    const uint32_t(&w1)[WPT] = wbuf[s][r][1];
                    float acc[MT][4];
                    if constexpr (BITS == 4) {
#pragma unroll
                        for (int j = 0; j < STEPS; ++j) {
                            const int q = j >> 1, sh = (j & 1) * 8;
                            uint32_t a[4];
                            a[0] = and_or(w0[q] >> sh, MASK, MAGIC);
                            a[1] = and_or(w1[q] >> sh, MASK, MAGIC);
                            a[2] = and_or(w0[q] >> (sh + 4), MASK, MAGIC);
                            a[3] = and_or(w1[q] >> (sh + 4), MASK, MAGIC);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                if (j == 0) mma16816<F16>(acc[mt], a, bf[mt][j][0], bf[mt][j][1], zero4);
                                else mma16816<F16>(acc[mt], a, bf[mt][j][0], bf[mt][j][1], acc[mt]);
                            }
                        }
                    } else {
                        float acc_hi[MT][4];
#pragma unroll
                        for (int j = 0; j < STEPS; ++j) {
                            uint32_t alo[4], ahi[4];
                            alo[0] = and_or(w0[j], MASK, MAGIC);
                            alo[1] = and_or(w1[j], MASK, MAGIC);
                            alo[2] = and_or(w0[j] >> 8, MASK, MAGIC);
                            alo[3] = and_or(w1[j] >> 8, MASK, MAGIC);
                            ahi[0] = and_or(w0[j] >> 4, MASK, MAGIC);
                            ahi[1] = and_or(w1[j] >> 4, MASK, MAGIC);
                            ahi[2] = and_or(w0[j] >> 12, MASK, MAGIC);
                            ahi[3] = and_or(w1[j] >> 12, MASK, MAGIC);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                if (j == 0) {
                                    mma16816<F16>(acc[mt], alo, bf[mt][j][0], bf[mt][j][1], zero4);
                                    mma16816<F16>(acc_hi[mt], ahi, bf[mt][j][0], bf[mt][j][1], zero4);
                                } else {
                                    mma16816<F16>(acc[mt], alo, bf[mt][j][0], bf[mt][j][1], acc[mt]);
                                    mma16816<F16>(acc_hi[mt], ahi, bf[mt][j][0], bf[mt][j][1], acc_hi[mt]);
                                }
                            }
                        }
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int c = 0; c < 4; ++c) acc[mt][c] = fmaf(16.0f, acc_hi[mt][c], acc[mt][c]);
                    }
                    // y += s * acc + (b - OFF_TOTAL * s) * sum(x)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const float sv = s_[r][h];
                        const float bv = fmaf(-OFF_TOTAL, sv, b_[r][h]);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int c2 = 0; c2 < 2; ++c2) {
                                const int c = 2 * h + c2;
                                res[r][mt][c] = fmaf(sv, acc[mt][c], fmaf(bv, xs[mt][c], res[r][mt][c]));
                            }
                    }
                }
            }
        }
    }

    // ---- fixed-order reduction of the K slices -----------------------------
    constexpr int NV = RW * MT * 4;
    extern __shared__ float red[];  // [nwarps][NV][32]
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) red[((warp * NV) + (r * MT + mt) * 4 + c) * 32 + lane] = res[r][mt][c];
    __syncthreads();
    for (int idx = threadIdx.x; idx < NV * 32; idx += blockDim.x) {
        const int ln = idx & 31, v = idx >> 5;
        float sum = 0.0f;
        for (int wk = 0; wk < nwarps; ++wk) sum += red[(wk * NV + v) * 32 + ln];
        const int c = v & 3, mt = (v >> 2) % MT, r = (v >> 2) / MT;
        const int gg = ln >> 2, tt = ln & 3;
        const int n = n_block + 16 * r + gg + 8 * (c >> 1);
        const int m = 8 * mt + 2 * tt + (c & 1);
        if (n < N && m < m_count) {
            long long dst = r0 + m;
            if constexpr (GATHER) {
                if (args.seg.row_scale != nullptr) sum *= __ldg(args.seg.row_scale + r0 + m);
                if (args.seg.row_dst != nullptr) dst = __ldg(args.seg.row_dst + r0 + m);
                if (dst < 0 || dst >= args.seg.y_rows) continue;
            }
            args.y[dst * N + n] = H::from_f32(sum);
        }
    }
}

}  // namespace qmm

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace qmm_host {

using qmm::QmvArgs;

// The K-split warp count depends on (N, K) only, never on M, so an M-row call
// reduces every row in exactly the order of a single-row call.
int qmv_k_warps(long long N, long long K, int gs) {
    const long long G = K / (gs < 64 ? gs : 64);  // K chunks
    const int rw = N > 4096 ? 2 : 1;
    const long long ctas = (N + 16 * rw - 1) / (16 * rw);
    long long want = (148LL * 16 + ctas - 1) / ctas;  // ~16 resident warps per SM
    if (want > 16) want = 16;
    long long cap = G / 2 > 0 ? G / 2 : 1;  // at least two chunks per warp
    if (want > cap) want = cap;
    if (want < 1) want = 1;
    return (int)want;
}

int qmv_rows_per_warp(long long N) { return N > 4096 ? 2 : 1; }

template <int BITS, int GS, bool F16, int MT, int RW, bool GATHER>
static int launch_qmv_t(const QmvArgs& a, int k_warps, int grid_y, cudaStream_t st) {
    // prefetch depth: about 32 registers of packed words in flight per thread
    constexpr int WREGS = RW * 2 * qmm::QGeom<BITS, GS>::WPT;
    constexpr int PD = 32 / WREGS < 2 ? 2 : (32 / WREGS > 8 ? 8 : 32 / WREGS);
    auto kern = qmm::qmv_kernel<BITS, GS, F16, MT, RW, PD, GATHER>;
    const int threads = 32 * k_warps;
    const size_t smem = (size_t)k_warps * RW * MT * 4 * 32 * sizeof(float);
    dim3 grid((unsigned)((a.N + 16 * RW - 1) / (16 * RW)), (unsigned)grid_y, 1);
    kern<<<grid, threads, smem, st>>>(a);
    return cuda_status(cudaGetLastError(), "qmv launch");
}

template <int BITS, int GS, bool F16, bool GATHER>
static int launch_qmv_mt(const QmvArgs& a, int mt, int rw, int k_warps, int grid_y, cudaStream_t st) {
    if (mt == 1) {
        return rw == 1 ? launch_qmv_t<BITS, GS, F16, 1, 1, GATHER>(a, k_warps, grid_y, st)
                       : launch_qmv_t<BITS, GS, F16, 1, 2, GATHER>(a, k_warps, grid_y, st);
    }
    return rw == 1 ? launch_qmv_t<BITS, GS, F16, 2, 1, GATHER>(a, k_warps, grid_y, st)
                   : launch_qmv_t<BITS, GS, F16, 2, 2, GATHER>(a, k_warps, grid_y, st);
}

template <bool GATHER>
int launch_qmv(const QmvArgs& a, int bits, int gs, bool f16, int mt, int rw, int k_warps, int grid_y,
               cudaStream_t st) {
#define QMM_QMV_CASE(B, S)                                                                               \
    if (bits == B && gs == S)                                                                             \
        return f16 ? launch_qmv_mt<B, S, true, GATHER>(a, mt, rw, k_warps, grid_y, st)                   \
                   : launch_qmv_mt<B, S, false, GATHER>(a, mt, rw, k_warps, grid_y, st);
    QMM_QMV_CASE(4, 32)
    QMM_QMV_CASE(4, 64)
    QMM_QMV_CASE(4, 128)
    QMM_QMV_CASE(8, 32)
    QMM_QMV_CASE(8, 64)
    QMM_QMV_CASE(8, 128)
#undef QMM_QMV_CASE
    set_error("qmv: bits=%d group_size=%d not supported", bits, gs);
    return QMM_EUNSUPPORTED;
}

template int launch_qmv<false>(const QmvArgs&, int, int, bool, int, int, int, int, cudaStream_t);
template int launch_qmv<true>(const QmvArgs&, int, int, bool, int, int, int, int, cudaStream_t);

}  // namespace qmm_host
