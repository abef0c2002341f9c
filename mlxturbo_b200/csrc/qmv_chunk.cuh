// qmv_chunk.cuh -- the per-chunk arithmetic of the decode kernels (qmv.cu):
// one 64-value (or 32-value) K chunk of RW 16-row weight tiles against up to
// 16 activation rows on warp-level tensor-core MMA.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace qmm {

// The K loop walks "chunks" of CH = min(group_size, 64) values; a 128-wide
// quantisation group is two chunks sharing one scale and bias.
// Set when a bounded wait in a decode kernel gave up (one flag per translation unit).
static __device__ int g_qmv_error;

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

// Activation loads are volatile so the compiler keeps them where they are
// issued (a chunk ahead of their use) instead of sinking them under register
// pressure.
template <int XR>
QMM_DEVINL void load_x(uint32_t (&dst)[XR], const uint16_t* p, bool valid) {
#pragma unroll
    for (int i = 0; i < XR; i += 4) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (valid) v = ld_v4(p + 2 * i);  // x: an earlier kernel's output
        dst[i] = v.x;
        dst[i + 1] = v.y;
        dst[i + 2] = v.z;
        dst[i + 3] = v.w;
    }
}

// Shared-memory layout of one warp's TMA ring: STG stages of 16*RW rows x
// 128 bytes (one 128-byte swizzle span of packed words per row).
template <int BITS, int GS, int RW, int STG_ = 0>
struct QRing {
    using G_ = QGeom<BITS, GS>;
    static constexpr int ROWS = 16 * RW;
    static constexpr int CHUNK_BYTES = G_::CH * BITS / 8;  // packed bytes of one chunk of one row
    static constexpr int CPS = 128 / CHUNK_BYTES;          // chunks per stage
    static constexpr int STAGE_BYTES = ROWS * 128;
    static constexpr int STG = STG_ ? STG_ : (RW == 1 ? 4 : 2);  // stages per warp (8 KB in flight per warp)
    static constexpr int WARP_BYTES = STG * STAGE_BYTES;
};

// Shared-memory loads of WPT packed words at a 32-bit shared address plus a
// compile-time byte offset (keeps the per-row offsets out of the ALU).
template <int WPT, int IMM>
QMM_DEVINL void lds_words(uint32_t addr, uint32_t* d) {
    if constexpr (WPT == 1) {
        asm volatile("ld.shared.u32 %0, [%1+%2];" : "=r"(d[0]) : "r"(addr), "n"(IMM));
    } else if constexpr (WPT == 2) {
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(d[0]), "=r"(d[1]) : "r"(addr), "n"(IMM));
    } else {
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4+%5];"
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                     : "r"(addr), "n"(IMM));
    }
}

template <int RW, int WPT, int R = 0>
QMM_DEVINL void lds_tile_rows(uint32_t addr, uint32_t (&wv)[RW][2][WPT]) {
    if constexpr (R < RW) {
        lds_words<WPT, (16 * R) * 128>(addr, wv[R][0]);
        lds_words<WPT, (16 * R + 8) * 128>(addr, wv[R][1]);
        lds_tile_rows<RW, WPT, R + 1>(addr, wv);
    }
}

// f(integral_constant<0>), ..., f(integral_constant<N_-1>): a loop over
// compile-time chunk indices.
template <int I, int N_, class F>
QMM_DEVINL void unroll_chunks_impl(F&& f) {
    if constexpr (I < N_) {
        f(std::integral_constant<int, I>{});
        unroll_chunks_impl<I + 1, N_>(f);
    }
}
template <int N_, class F>
QMM_DEVINL void unroll_chunks(F&& f) {
    unroll_chunks_impl<0, N_>(f);
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

// res[r][mt] += s * sum(q*x) + b * sum(x) for one chunk:
//   xr   activations of the chunk (thread's B-fragment values per MMA n-tile)
//   wv   packed words of rows g, g+8 of each tile
//   s_/b_ the chunk group's scale and bias of rows g, g+8 of each tile
template <int BITS, bool F16, int MT, int RW, int XR, int WPT, int STEPS>
QMM_DEVINL void chunk_math(float (&res)[RW][MT][4], const uint32_t (&xr)[MT][XR], const uint32_t (&wv)[RW][2][WPT],
                           const float (&s_)[RW][2], const float (&b_)[RW][2]) {
    using H = Half<F16>;
    constexpr uint32_t MAGIC = H::kMagic;
    constexpr uint32_t MASK = 0x000F000Fu;
    // sum(q*x) = acc - OFF_TOTAL * sum(x) with the code offsets folded.
    constexpr float OFF = H::kOffset;
    constexpr float OFF_TOTAL = BITS == 4 ? OFF : 17.0f * OFF;
    const uint32_t ones[4] = {H::kOne2, H::kOne2, H::kOne2, H::kOne2};
    const float zero4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    // Step-major issue: at every k16 step the sum(x) chain and all
    // row-tile chains advance together, so RW*MT (+MT) independent
    // MMAs are in flight instead of one dependent chain at a time.
    float xs[MT][4];
    float acc[RW][MT][4];
    float acc_hi[BITS == 8 ? RW : 1][MT][4];
#pragma unroll
    for (int j = 0; j < STEPS; ++j) {
        uint32_t bf[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            x_frag<BITS, XR>(xr[mt], j, bf[mt][0], bf[mt][1]);
            if (j == 0) mma16816<F16>(xs[mt], ones, bf[mt][0], bf[mt][1], zero4);
            else mma16816<F16>(xs[mt], ones, bf[mt][0], bf[mt][1], xs[mt]);
        }
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            const uint32_t(&w0)[WPT] = wv[r][0];
            const uint32_t(&w1)[WPT] = wv[r][1];
            if constexpr (BITS == 4) {
                const int q = j >> 1, sh = (j & 1) * 8;
                uint32_t a[4];
                a[0] = and_or(w0[q] >> sh, MASK, MAGIC);
                a[1] = and_or(w1[q] >> sh, MASK, MAGIC);
                a[2] = and_or(w0[q] >> (sh + 4), MASK, MAGIC);
                a[3] = and_or(w1[q] >> (sh + 4), MASK, MAGIC);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    if (j == 0) mma16816<F16>(acc[r][mt], a, bf[mt][0], bf[mt][1], zero4);
                    else mma16816<F16>(acc[r][mt], a, bf[mt][0], bf[mt][1], acc[r][mt]);
                }
            } else {
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
                        mma16816<F16>(acc[r][mt], alo, bf[mt][0], bf[mt][1], zero4);
                        mma16816<F16>(acc_hi[r][mt], ahi, bf[mt][0], bf[mt][1], zero4);
                    } else {
                        mma16816<F16>(acc[r][mt], alo, bf[mt][0], bf[mt][1], acc[r][mt]);
                        mma16816<F16>(acc_hi[r][mt], ahi, bf[mt][0], bf[mt][1], acc_hi[r][mt]);
                    }
                }
            }
        }
    }
    // y += s * acc + (b - OFF_TOTAL * s) * sum(x)
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        if constexpr (BITS == 8) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int c2 = 0; c2 < 4; ++c2)
                    acc[r][mt][c2] = fmaf(16.0f, acc_hi[r][mt][c2], acc[r][mt][c2]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float svv = s_[r][h];
            const float bvv = fmaf(-OFF_TOTAL, svv, b_[r][h]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    const int cc = 2 * h + c2;
                    res[r][mt][cc] = fmaf(svv, acc[r][mt][cc], fmaf(bvv, xs[mt][cc], res[r][mt][cc]));
                }
        }
    }
}

}  // namespace qmm
