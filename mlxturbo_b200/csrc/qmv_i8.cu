// qmv_i8.cu -- decode / verify (M <= 8 activation rows) on warp-level
// integer MMA: the stream-K schedule of qmv_sk.cu with integer arithmetic.
//
// Same problem as qmv_sk.cu (y[m, n] = sum_k x[m, k] * (s * q + b)), same
// schedule (a fixed number of warps each streaming an equal contiguous range
// of (32-row tile, K stage) units through a per-warp TMA ring), a different
// split-tile sum (the tile's first owner adds the later owners' partials,
// published as epoch-tagged words, in warp order) and different per-chunk
// arithmetic:
//
//   A = the codes as u8 in mma.sync.m16n8k32 fragments.  A thread's packed
//       word w feeds one k32 step of one row: 4-bit codes as
//       (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F) -- three integer ops per 8
//       weights; 8-bit codes as the words themselves.
//   B = the activations as two exact int8 planes per quantisation group
//       (X = rint(x * 2^(140 - e)) = 128 * d1 + d0 with e the group's largest
//       f32 exponent; values within 2^6 of the group maximum are exact), one
//       n8 column per (row, plane).  A prep kernel writes them once per call
//       already in the fragment register layout, with each chunk's sum of x
//       and 2^(e - 140), so the main loop loads one 8-byte fragment per
//       (k32 step, n-tile) and no activation arithmetic remains in it.
//   Per chunk and row: y += s * 2^(e - 140) * (128 * D1 + D0) + b * sum(x),
//       D exact in s32, 128 * D1 + D0 formed in s32 and converted once.
//
// Rows of an M-row call are computed independently (their own columns and
// terms), so each has the bits of a single-row call.

#include <stdlib.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "qmv_chunk.cuh"
#include "tc.cuh"
#include "tma.cuh"

namespace qmm {

__device__ int g_i8_error;

template <int BITS, int GS, int MP>
struct I8Geom {
    using G_ = QGeom<BITS, GS>;
    static constexpr int CH = G_::CH;                // K values per chunk
    static constexpr int WPT = G_::WPT;              // packed words per thread per chunk per row
    static constexpr int STEPS = CH / 32;            // k32 MMA steps per chunk
    static constexpr int CPG = GS / CH;              // chunks per group
    static constexpr int NT = MP <= 4 ? 1 : 2;       // n8 tiles: two planes of four rows each
    static constexpr int FRAG_CHUNK = STEPS * NT * 32 * 8;  // fragment bytes per chunk
    static_assert(STEPS >= 1 && (BITS == 4 ? WPT == STEPS : WPT == 2 * STEPS), "word / step geometry");
};

struct I8Args {
    uint16_t* y;
    int M, N, K;
    int Ut;             // K stages per tile
    int T;              // row tiles of 32 rows
    int warps_total;    // warps launched
    unsigned long long* tslots;  // [warps_total][32 lanes][8]: (epoch << 32 | partial) words
    const uint32_t* epoch;       // this call's epoch (the prep kernel advances it)
    const uint8_t* frag;  // [chunks][STEPS][NT][32 lanes][2 x u32] activation fragments
    const float2* terms;  // [chunks][MP]: (sum of x over the chunk, 2^(e - 140) of its group)
    // fused greedy sampling (null: off): per activation row, the maximum of
    // argmax_key(stored logit, n_offset + n) over the outputs, by atomicMax
    unsigned long long* amax;
    long long n_offset;
};

// Order-preserving key of a (logit, index) pair: larger logits give larger
// keys, and equal logits the smaller index (the first occurrence, as a
// single-device argmax returns).  The logit is the value as stored (rounded to
// the output dtype).
QMM_DEVINL unsigned long long argmax_key(float f, long long n) {
    const uint32_t u = f == 0.0f ? 0u : __float_as_uint(f);  // -0 ties with +0, as in argmax
    const uint32_t mono = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)mono << 32) | (0xFFFFFFFFu - (uint32_t)n);
}

QMM_DEVINL void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Prep: one warp (one CTA) per quantisation group, all activation rows.
//
// Lane (g, t) writes its own 8-byte fragment of k32 step j of n-tile nt:
// column g is activation row m = 4 * nt + g / 2, plane g % 2, and the 8 bytes
// are the planes of the 8 consecutive K values kc0 .. kc0 + 7 of the chunk,
// kc0 = (t * STEPS + j) * 8:
//   4-bit codes: register 0 holds values 0, 2, 4, 6 and register 1 values
//                1, 3, 5, 7 (the nibble order of a packed word: its even
//                nibbles feed A register 0, its odd nibbles A register 2);
//   8-bit codes: register 0 holds values 0..3, register 1 values 4..7.
// The four lanes t of a column hold the group's values of one row, so the
// group maximum and the chunk sums are two shuffles away.  Columns of rows
// M..MP-1 are written as zeros.
// ---------------------------------------------------------------------------
template <int BITS, int GS, bool F16, int MP>
__global__ void __launch_bounds__(32) qmv_i8_prep_kernel(const uint16_t* x, int M, int K, int x16, uint8_t* frag,
                                                         float2* terms, uint32_t* epoch) {
    using I = I8Geom<BITS, GS, MP>;
    using H = Half<F16>;
    constexpr int STEPS = I::STEPS, CPG = I::CPG, NT = I::NT, CH = I::CH;
    pdl_launch_dependents();
    pdl_wait();  // x is the previous kernel's output (and the previous call is complete)
    const int q = blockIdx.x, lane = threadIdx.x, g = lane >> 2, t = lane & 3;
    // a new epoch per call: partial sums tagged with it cannot be mistaken for
    // an earlier call's (CUDA graph replays included)
    if (q == 0 && lane == 0) *epoch = *epoch + 1u;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int m = 4 * nt + (g >> 1), p = g & 1;
        const bool valid = m < M;
        uint32_t v[CPG][STEPS][4];  // 8 values (bf16 / f16 pairs) per (chunk, step)
        const uint16_t* xr = x + (size_t)(valid ? m : 0) * K + (size_t)q * GS + t * STEPS * 8;
#pragma unroll
        for (int cl = 0; cl < CPG; ++cl)
#pragma unroll
            for (int j = 0; j < STEPS; ++j) {
                const uint16_t* src = xr + cl * CH + j * 8;
                if (!valid) {
                    v[cl][j][0] = v[cl][j][1] = v[cl][j][2] = v[cl][j][3] = 0u;
                } else if (x16) {
                    const uint4 u = ld_v4(src);
                    v[cl][j][0] = u.x, v[cl][j][1] = u.y, v[cl][j][2] = u.z, v[cl][j][3] = u.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[cl][j][i] = (uint32_t)src[2 * i] | ((uint32_t)src[2 * i + 1] << 16);
                }
            }
        float amax = 0.0f;
        float csum[CPG];
#pragma unroll
        for (int cl = 0; cl < CPG; ++cl) {
            csum[cl] = 0.0f;
#pragma unroll
            for (int j = 0; j < STEPS; ++j)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float f = (i & 1) ? H::hi_f32(v[cl][j][i >> 1]) : H::lo_f32(v[cl][j][i >> 1]);
                    amax = fmaxf(amax, fabsf(f));
                    csum[cl] += f;
                }
        }
#pragma unroll
        for (int off = 1; off <= 2; off <<= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
#pragma unroll
            for (int cl = 0; cl < CPG; ++cl) csum[cl] += __shfl_xor_sync(0xffffffffu, csum[cl], off);
        }
        int e = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
        e = e < 14 ? 14 : e;  // tiny or zero groups use the smallest scale
        const float up = __uint_as_float((uint32_t)(267 - e) << 23);  // 2^(140 - e)
        const int sh = 7 * p;  // plane 0: bits 0..6 (d0); plane 1: bits 7..14 (the s8 pattern of d1)
        const uint32_t mask = valid ? (p ? 0xFFu : 0x7Fu) : 0u;
#pragma unroll
        for (int cl = 0; cl < CPG; ++cl) {
            const size_t chunk = (size_t)q * CPG + cl;
#pragma unroll
            for (int j = 0; j < STEPS; ++j) {
                uint32_t b[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    // X = rint(x * 2^(140-e)) rides in the low bits of 1.5 * 2^23 + X
                    const float f = (i & 1) ? H::hi_f32(v[cl][j][i >> 1]) : H::lo_f32(v[cl][j][i >> 1]);
                    b[i] = (__float_as_uint(fmaf(f, up, 12582912.0f)) >> sh) & mask;
                }
                uint32_t r0, r1;
                if constexpr (BITS == 4) {
                    r0 = b[0] | (b[2] << 8) | (b[4] << 16) | (b[6] << 24);
                    r1 = b[1] | (b[3] << 8) | (b[5] << 16) | (b[7] << 24);
                } else {
                    r0 = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
                    r1 = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
                }
                *reinterpret_cast<uint2*>(frag + chunk * I::FRAG_CHUNK + ((size_t)(j * NT + nt) * 32 + lane) * 8) =
                    make_uint2(r0, r1);
            }
            if (p == 0 && t == 0 && m < MP)  // terms hold MP rows; columns of rows >= MP exist only in the fragments
                terms[chunk * MP + m] =
                    valid ? make_float2(csum[cl], __uint_as_float((uint32_t)(e - 13) << 23)) : make_float2(0.0f, 0.0f);
        }
    }
}

// ---------------------------------------------------------------------------
// Main kernel: 4 warps per CTA, each a stream-K worker with its own ring.
// ---------------------------------------------------------------------------
constexpr int kI8Warps = 4;
constexpr int kI8SpinLimit = 1 << 22;  // polls of a peer's partial (~0.5 s) before the call reports an error

template <int BITS, int GS, bool F16, int MP, int RING>
__global__ void __launch_bounds__(32 * kI8Warps, 4)
    qmv_i8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                  const __grid_constant__ CUtensorMap bmap, I8Args a) {
    using I = I8Geom<BITS, GS, MP>;
    constexpr int RW = 2;
    using R_ = QRing<BITS, GS, RW, RING>;
    using H = Half<F16>;
    constexpr int WPT = I::WPT, STEPS = I::STEPS, NT = I::NT, CH = I::CH, CPG = I::CPG;
    constexpr int CPS = R_::CPS, STG = R_::STG, ROWS = R_::ROWS;
    constexpr int CBU = R_::CHUNK_BYTES / 16;
    constexpr int NV = RW * NT * 2;  // partial values per lane
    static_assert(NV <= 8 && NV % 2 == 0, "slot size");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int N = a.N;
    const int gw = blockIdx.x * nwarps + warp;

    constexpr int SC_BYTES = ROWS * 16;  // one 8-group box of scales (or biases) per stage
    uint8_t* sring = smem + nwarps * R_::WARP_BYTES + warp * (STG * 2 * SC_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + nwarps * (R_::WARP_BYTES + STG * 2 * SC_BYTES));
    volatile int* abort = reinterpret_cast<volatile int*>(bars + nwarps * STG) + warp;
    const uint32_t bar0 = smem_u32(bars + warp * STG);
    const uint32_t ring0 = smem_u32(smem + warp * R_::WARP_BYTES);

    pdl_launch_dependents();
    if (lane == 0) {
        *abort = 0;
        for (int s = 0; s < STG; ++s) mbar_init(bar0 + 8 * s, 1);
        mbar_fence_init();
    }
    __syncwarp();

    const long long total = (long long)a.T * a.Ut;
    const int wt = total < a.warps_total ? (int)total : a.warps_total;
    if (gw >= wt) return;  // no unit for this warp (no barrier below spans warps)
    const long long ua = total * gw / wt, ub = total * (gw + 1) / wt;
    const int nst = (int)(ub - ua);

    // The issue state advances in every lane (warp-uniform values) and one
    // elected lane issues the copies: issue from a lane-0 branch works on
    // non-uniform registers and costs more per copy.
    int i_tile = (int)(ua / a.Ut), i_ku = (int)(ua - (long long)i_tile * a.Ut);
    auto issue_w = [&](int s) {
        const int wrow = i_tile * ROWS, ku = i_ku;
        if (++i_ku == a.Ut) {
            i_ku = 0;
            ++i_tile;
        }
        // groups of this stage start at ku*CPS/CPG; the box starts at the
        // 8-group (16-byte) boundary below and the kernel indexes past it
        const int gx = (ku * (CPS / CPG)) & ~7;
        const uint32_t sdst = smem_u32(sring) + s * 2 * SC_BYTES;
        if (elect_one()) {
            mbar_expect_tx(bar0 + 8 * s, R_::STAGE_BYTES + 2 * SC_BYTES);
            tma_load_2d(ring0 + s * R_::STAGE_BYTES, &wmap, bar0 + 8 * s, ku * CPS * (CH * BITS / 32), wrow);
            tma_load_2d(sdst, &smap, bar0 + 8 * s, gx, wrow);
            tma_load_2d(sdst + SC_BYTES, &bmap, bar0 + 8 * s, gx, wrow);
        }
        __syncwarp();
    };
    if (lane == 0) {
        tma_prefetch_desc(&wmap);
        tma_prefetch_desc(&smap);
        tma_prefetch_desc(&bmap);
    }
    for (int s = 0; s < STG && s < nst; ++s) issue_w(s);  // weights do not depend on the previous kernel
    pdl_wait();  // the activation fragments (and y's readers) belong to earlier kernels
    const uint32_t E = *reinterpret_cast<const volatile uint32_t*>(a.epoch);

    const uint32_t tb = (uint32_t)t * WPT * 4;
    const uint32_t tconst = ((((tb >> 4) ^ (uint32_t)g) & (CBU - 1)) << 4) | (tb & 15);
    const uint32_t hkey = (uint32_t)g & 7u & ~(uint32_t)(CBU - 1);
    const uint32_t rowbase = (uint32_t)g * 128;

    float res[RW][NT][2];
    int cur_tile = -1, seg_k0 = 0;

    auto flush = [&](int tile, int k0, int k1) {
        const bool whole = (k0 == 0 && k1 == a.Ut);
        float out[RW][NT][2];
        bool store = whole;
        float* rr = &res[0][0][0];
        float* oo = &out[0][0][0];
        if (!whole) {
            // A split tile is summed by its first owner f, in owner order
            // f, f+1, ..., l.  The tile is f's last work; every later owner's
            // range starts inside it, so each warp publishes at most one
            // partial (its first tile's) and sums at most one tile (its last).
            // A partial travels as 64-bit (epoch << 32 | value) words: one
            // store publishes value and tag together, and the first owner
            // polls them, with a bound, instead of a counter round trip.
            const long long u0 = (long long)tile * a.Ut;
            const int f = (int)(((u0 + 1) * wt - 1) / total), l = (int)(((u0 + a.Ut) * wt - 1) / total);
            // slot of warp w: [activation row m < MP][tile row n 0..31] words
            if (gw != f) {
                unsigned long long* my = a.tslots + (size_t)gw * 256;
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int m = 4 * nt + t;
                            if (m < a.M) {
                                const unsigned long long wd =
                                    ((unsigned long long)E << 32) | __float_as_uint(res[r][nt][h]);
                                asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(my + m * 32 + 16 * r + 8 * h + g),
                                             "l"(wd)
                                             : "memory");
                            }
                        }
            } else {
                // lane = tile row n: own partials moved there by shuffles
                // (lane 4 * (n % 8) + m % 4 holds (n, m) at [n / 16][m / 4][(n / 8) % 2])
                const int rs = lane >> 4, hs = (lane >> 3) & 1, gs_ = lane & 7;
                float acc[MP];
#pragma unroll
                for (int m = 0; m < MP; ++m) {
                    const int src = 4 * gs_ + (m & 3), nt = m >> 2;
                    const float v00 = __shfl_sync(0xffffffffu, res[0][nt][0], src);
                    const float v01 = __shfl_sync(0xffffffffu, res[0][nt][1], src);
                    const float v10 = __shfl_sync(0xffffffffu, res[1][nt][0], src);
                    const float v11 = __shfl_sync(0xffffffffu, res[1][nt][1], src);
                    acc[m] = rs == 0 ? (hs == 0 ? v00 : v01) : (hs == 0 ? v10 : v11);
                }
                // the later owners' partials, PB owners per batch of loads (one round trip each)
                constexpr int PB = MP >= 8 ? 1 : 16 / MP;  // <= 16 words in flight per lane
                for (int p0 = f + 1; p0 <= l; p0 += PB) {
                    unsigned long long q[PB][MP];
                    for (int spin = 0;; ++spin) {
#pragma unroll
                        for (int i = 0; i < PB; ++i)
#pragma unroll
                            for (int m = 0; m < MP; ++m) {
                                q[i][m] = (unsigned long long)E << 32;
                                if (p0 + i <= l && m < a.M)
                                    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];"
                                                 : "=l"(q[i][m])
                                                 : "l"(a.tslots + (size_t)(p0 + i) * 256 + m * 32 + lane)
                                                 : "memory");
                            }
                        bool ok = true;
#pragma unroll
                        for (int i = 0; i < PB; ++i)
#pragma unroll
                            for (int m = 0; m < MP; ++m) ok = ok && (uint32_t)(q[i][m] >> 32) == E;
                        if (__all_sync(0xffffffffu, ok)) break;
                        if (spin >= kI8SpinLimit) {  // a peer never published: report, do not hang
                            if (lane == 0) atomicOr(&g_i8_error, 2);
                            break;
                        }
                        __nanosleep(64);
                    }
#pragma unroll
                    for (int i = 0; i < PB; ++i)
#pragma unroll
                        for (int m = 0; m < MP; ++m)
                            if (p0 + i <= l) acc[m] += __uint_as_float((uint32_t)q[i][m]);
                }
                const int n = tile * ROWS + lane;
#pragma unroll
                for (int m = 0; m < MP; ++m) {
                    const uint16_t v = H::from_f32(acc[m]);
                    if (m < a.M && n < N) a.y[(long long)m * N + n] = v;
                    if (a.amax) {  // this tile's largest key of row m, one atomic per warp
                        unsigned long long key = (m < a.M && n < N) ? argmax_key(H::to_f32(v), a.n_offset + n) : 0ull;
#pragma unroll
                        for (int o = 16; o >= 1; o >>= 1) {
                            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                            key = k2 > key ? k2 : key;
                        }
                        if (lane == 0 && m < a.M) atomicMax(a.amax + m, key);
                    }
                }
            }
        } else {
#pragma unroll
            for (int v = 0; v < NV; ++v) oo[v] = rr[v];
        }
        if (store) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int m = 4 * nt + t;
                unsigned long long key = 0ull;
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int n = tile * ROWS + 16 * r + 8 * h + g;
                        const uint16_t v = H::from_f32(out[r][nt][h]);
                        if (n < N && m < a.M) {
                            a.y[(long long)m * N + n] = v;
                            const unsigned long long k = argmax_key(H::to_f32(v), a.n_offset + n);
                            key = k > key ? k : key;
                        }
                    }
                if (a.amax) {  // lanes of one row m share t: reduce over g, one atomic per (warp, row)
#pragma unroll
                    for (int o = 4; o <= 16; o <<= 1) {
                        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
                        key = k2 > key ? k2 : key;
                    }
                    if (g == 0 && m < a.M) atomicMax(a.amax + m, key);
                }
            }
        }
    };

    // activation fragments and per-chunk terms of chunk cg, one chunk ahead
    uint2 bf[2][STEPS][NT];
    float2 tm[2][NT];
    auto fetch = [&](int B, int cg) {
        const uint2* fp = reinterpret_cast<const uint2*>(a.frag + (size_t)cg * I::FRAG_CHUNK) + lane;
#pragma unroll
        for (int j = 0; j < STEPS; ++j)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) bf[B][j][nt] = ld_dep(fp + (j * NT + nt) * 32);  // the prep kernel's output
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) tm[B][nt] = ld_dep(a.terms + (size_t)cg * MP + (4 * nt + t < MP ? 4 * nt + t : 0));
    };
    uint32_t sbw[RW][2][2];  // (scale, bias) pairs of two groups
    int m_tile = (int)(ua / a.Ut), m_ku = (int)(ua - (long long)m_tile * a.Ut);
    const int C = a.K / CH;
    for (int st = 0; st < nst; ++st) {
        const int tile = m_tile, ku = m_ku;
        if (++m_ku == a.Ut) {
            m_ku = 0;
            ++m_tile;
        }
        if (tile != cur_tile) {
            cur_tile = tile;
            seg_k0 = ku;
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) res[r][nt][0] = res[r][nt][1] = 0.0f;
            fetch(0, ku * CPS);
        }
        const bool next_same_tile = (ku + 1 < a.Ut) && (st + 1 < nst);
        const int s = st % STG;
        mbar_wait_bounded(bar0 + 8 * s, (uint32_t)(st / STG) & 1u, abort, &g_i8_error);
        const uint32_t stage_addr = ring0 + s * R_::STAGE_BYTES + rowbase;
        const bool full = (ku + 1) * CPS <= C;
        auto do_chunk = [&](auto cc, auto fullc) {
            constexpr int c = decltype(cc)::value;
            constexpr bool FULL = decltype(fullc)::value;
            constexpr int B = c & 1;
            if constexpr (c + 1 < CPS) {
                if (FULL || ku * CPS + c + 1 < C) fetch(B ^ 1, ku * CPS + c + 1);
            } else {
                if (next_same_tile) fetch(B ^ 1, (ku + 1) * CPS);
            }
            float s_[RW][2], b_[RW][2];
            {
                constexpr int GPS = CPS / CPG, gq = c / CPG;
                const int gi = ((ku * GPS) & 7) + gq;
                const uint16_t* sp = reinterpret_cast<const uint16_t*>(sring + s * 2 * SC_BYTES) + g * 8;
                if constexpr (GPS % 2 == 0) {
                    if constexpr (c % CPG == 0 && gq % 2 == 0) {
#pragma unroll
                        for (int r = 0; r < RW; ++r)
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int row = 16 * r + 8 * h;
                                sbw[r][h][0] = *reinterpret_cast<const uint32_t*>(sp + row * 8 + gi);
                                sbw[r][h][1] = *reinterpret_cast<const uint32_t*>(sp + SC_BYTES / 2 + row * 8 + gi);
                            }
                    }
#pragma unroll
                    for (int r = 0; r < RW; ++r)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            s_[r][h] = (gq & 1) ? H::hi_f32(sbw[r][h][0]) : H::lo_f32(sbw[r][h][0]);
                            b_[r][h] = (gq & 1) ? H::hi_f32(sbw[r][h][1]) : H::lo_f32(sbw[r][h][1]);
                        }
                } else {
#pragma unroll
                    for (int r = 0; r < RW; ++r)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int row = 16 * r + 8 * h;
                            s_[r][h] = H::to_f32(sp[row * 8 + gi]);
                            b_[r][h] = H::to_f32(sp[SC_BYTES / 2 + row * 8 + gi]);
                        }
                }
            }
            uint32_t wv[RW][2][WPT];
            const uint32_t cofs = (((((uint32_t)(c * CBU)) ^ hkey) & 7u) << 4) | tconst;
            lds_tile_rows<RW, WPT>(stage_addr + cofs, wv);
            int acc[RW][NT][4];
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) acc[r][nt][0] = acc[r][nt][1] = acc[r][nt][2] = acc[r][nt][3] = 0;
#pragma unroll
            for (int j = 0; j < STEPS; ++j)
#pragma unroll
                for (int r = 0; r < RW; ++r) {
                    uint32_t af[4];
                    if constexpr (BITS == 4) {
                        af[0] = wv[r][0][j] & 0x0F0F0F0Fu;
                        af[1] = wv[r][1][j] & 0x0F0F0F0Fu;
                        af[2] = (wv[r][0][j] >> 4) & 0x0F0F0F0Fu;
                        af[3] = (wv[r][1][j] >> 4) & 0x0F0F0F0Fu;
                    } else {
                        af[0] = wv[r][0][2 * j];
                        af[1] = wv[r][1][2 * j];
                        af[2] = wv[r][0][2 * j + 1];
                        af[3] = wv[r][1][2 * j + 1];
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) imma16832(acc[r][nt], af, bf[B][j][nt].x, bf[B][j][nt].y);
                }
            // y += s * 2^(e-140) * (128 * D1 + D0) + b * sum(x)
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        // 128 * D1 + D0 in s32 (exact), then one conversion: exact for
                        // 4-bit codes (|v| < 2^24), within 2^-24 relative for 8-bit
                        const float dq = __int2float_rn(acc[r][nt][2 * h + 1] * 128 + acc[r][nt][2 * h]);
                        res[r][nt][h] = fmaf(s_[r][h] * tm[B][nt].y, dq, res[r][nt][h]);
                        res[r][nt][h] = fmaf(b_[r][h], tm[B][nt].x, res[r][nt][h]);
                    }
        };
        if (full) {
            unroll_chunks<CPS>([&](auto cc) { do_chunk(cc, std::true_type{}); });
        } else {
            unroll_chunks<CPS>([&](auto cc) {
                if (ku * CPS + decltype(cc)::value < C) do_chunk(cc, std::false_type{});
            });
        }
        __syncwarp();
        if (st + STG < nst) issue_w(s);
        if (ku == a.Ut - 1 || st == nst - 1) flush(tile, seg_k0, ku + 1);
    }
}

}  // namespace qmm

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace qmm_host {

size_t sk_workspace(long long M, long long N, long long K, int gs, int bits);

// Activation rows per n-tile layout: one row on its own; two to four rows share
// the four-row layout (measured on B200, HBM-cold: 17408x5120 at M = 2 takes
// 16.7 us with a two-row layout and 13.7 us with the four-row one, which M = 4
// also takes); five to eight take two n-tiles.  Rows keep their bits whatever
// the layout: each row has its own columns and terms.
static int i8_mp(int M) { return M <= 1 ? 1 : M <= 4 ? 4 : 8; }

// The workspace of qmm_quantized_matmul as this kernel uses it: the first
// 8 MiB stay the stream-K kernel's (counters, slots; this kernel touches
// none of it), then the epoch word, the tagged partial-sum slots (2 KiB per
// launched warp), the activation fragments and the per-chunk terms.  The
// region from 8 MiB on is this kernel's alone, at a fixed offset, so no
// other kernel's scratch of another shape lands on its slots; the epoch
// makes a slot from an earlier call read as not yet published.
constexpr size_t kI8Base = 8u << 20;
constexpr size_t kI8SlotBytes = 2048;                              // 32 lanes x 8 words
constexpr size_t kI8MaxWarps = 148 * (size_t)qmm::kI8Warps * 4;  // i8_plan launches at most this many
static size_t i8_sk_part(long long M, long long N, long long K, int gs, int bits) {
    (void)M, (void)N, (void)K, (void)gs, (void)bits;
    return kI8Base;
}
size_t i8_extra_workspace(long long M, long long K, int gs, int bits) {
    const int ch = gs < 64 ? gs : 64, mp = i8_mp((int)M), nt = mp <= 4 ? 1 : 2;
    const long long chunks = K / ch;
    (void)bits;
    return 1024 + kI8MaxWarps * kI8SlotBytes + (size_t)chunks * (ch / 32) * nt * 256 +
           ((size_t)chunks * mp * 8 + 1023) / 1024 * 1024;
}

// Whether the integer-MMA decode kernel takes this problem: M <= 8, K a
// multiple of the 128-byte stage, 16-byte scale rows (scales through TMA),
// and a matrix of at least 12 MiB of codes.  The size rule is the measured
// crossover on B200 (CUDA graphs with PDL, M = 1 / 4): 5120x6144 8.1 / 9.2 us
// against 10.7 / 11.4 us for the stream-K kernel, 6144x5120 8.1 / 8.7 against
// 9.4 / 9.6 us for the CTA-per-tile kernel, 4096x4096 (8 MiB) 6.3 / 7.4
// against 6.7 / 6.9 us and 1024x5120 6.1 against 4.3 us (the prep launch
// costs ~1 us); 17408x5120 13.7 against 17.4 us.  It depends on the matrix
// only, so every M <= 8 call on one matrix takes the same kernel and each row
// keeps the bits of a single-row call.
bool i8_supported(long long M, long long N, long long K, int gs, int bits, const void* sc, const void* bi) {
    if (M < 1 || M > 8 || (bits != 4 && bits != 8) || N < 1) return false;
    if (gs != 32 && gs != 64 && gs != 128) return false;
    if (K % (1024 / bits) != 0 || (K / gs) % 8 != 0) return false;
    if (((uintptr_t)sc | (uintptr_t)bi) & 15u) return false;
    return true;
}
bool i8_eligible(long long M, long long N, long long K, int gs, int bits, const void* sc, const void* bi) {
    return N * K * bits / 8 >= (12LL << 20) && i8_supported(M, N, K, gs, bits, sc, bi);
}

struct SkPlanI8 {
    int T, Ut, warps_total;
};

// Warps per CTA; the warps per SM stay 16 and the unit split (hence every
// sum's order) does not depend on it.  Smaller CTAs leave the SM in finer
// steps at the end of a launch, so the next kernel's CTAs move in and start
// their weight prefetch sooner: measured on B200 (CUDA graphs, PDL), 2-warp
// CTAs take the 7-projection decode layer from 72-74 to 68.5 us at M = 1
// (17408x5120: 13.2 against 13.6 us), while the 1.27 GB 8-bit lm_head
// streams better with 4-warp CTAs (234-238 against 253 us).
static int i8_wpc(long long code_bytes) { return code_bytes < (128LL << 20) ? 2 : qmm::kI8Warps; }

// Warps of CTAs of `wpc` warps with `smem` bytes of shared memory each that
// the current device holds at once, capped at 16 per SM (the design point) and
// at the slots the workspace provides.  The first owner of a split tile waits
// for the later owners' partials, so every warp of a launch must be able to be
// resident together: the grid never exceeds this count.  It depends on the
// device only (its SM count and the kernel's occupancy), cached per (kernel,
// device).
static int i8_resident_warps(const void* kern, int wpc, size_t smem) {
    struct Entry {
        const void* k;
        int dev, wpc, warps;
    };
    static Entry cache[64];
    static int n = 0;
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i)
        if (cache[i].k == kern && cache[i].dev == dev && cache[i].wpc == wpc) return cache[i].warps;
    int sms = 0, blocks = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kern, 32 * wpc, smem) != cudaSuccess) return 0;
    long long per_sm = (long long)blocks * wpc;
    if (per_sm > 16) per_sm = 16;
    long long w = (long long)sms * per_sm;
    if (w > (long long)kI8MaxWarps) w = (long long)kI8MaxWarps;
    if (n < 64) cache[n++] = Entry{kern, dev, wpc, (int)w};
    return (int)w;
}

static SkPlanI8 i8_plan(long long N, long long K, int gs, int bits, int max_warps) {
    SkPlanI8 p;
    const int ch = gs < 64 ? gs : 64, cps = 128 / (ch * bits / 8);
    p.T = (int)((N + 31) / 32);
    p.Ut = (int)((K / ch + cps - 1) / cps);
    const long long total = (long long)p.T * p.Ut;
    long long wt = (long long)max_warps;
    if (wt > total) wt = total >= qmm::kI8Warps ? total / qmm::kI8Warps * qmm::kI8Warps : total;
    p.warps_total = (int)wt;
    return p;
}

template <int BITS, int GS, bool F16, int MP, int RING>
static int launch_i8_t(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                       int M, int N, int K, void* ws, size_t ws_bytes, cudaStream_t st, unsigned long long* amax,
                       long long n_offset) {
    using I = qmm::I8Geom<BITS, GS, MP>;
    using R_ = qmm::QRing<BITS, GS, 2, RING>;
    auto kern = qmm::qmv_i8_kernel<BITS, GS, F16, MP, RING>;
    auto prep = qmm::qmv_i8_prep_kernel<BITS, GS, F16, MP>;
    const int wpc = i8_wpc((long long)N * K * BITS / 8);
    constexpr size_t SC = (size_t)R_::STG * 2 * R_::ROWS * 16;
    auto smem_for = [&](int w_) { return (size_t)w_ * (R_::WARP_BYTES + SC) + w_ * R_::STG * 8 + w_ * 4 + 1024; };
    int rc0 = ensure_smem_limit((const void*)kern, (int)smem_for(qmm::kI8Warps), "qmv_i8 smem attribute");
    if (rc0) return rc0;
    const int resident = i8_resident_warps((const void*)kern, wpc, smem_for(wpc));
    if (resident < 1) {
        set_error("qmv_i8: no resident CTA of %d warps on this device", wpc);
        return QMM_EUNSUPPORTED;
    }
    const SkPlanI8 p = i8_plan(N, K, GS, BITS, resident);
    if (p.T > 65536) {
        set_error("qmv_i8: N=%d needs %d row tiles", N, p.T);
        return QMM_EUNSUPPORTED;
    }
    const size_t base = i8_sk_part(M, N, K, GS, BITS);
    if (ws_bytes < base + i8_extra_workspace(M, K, GS, BITS)) {
        set_error("qmv_i8: workspace %zu < %zu bytes", ws_bytes, base + i8_extra_workspace(M, K, GS, BITS));
        return QMM_EINVAL;
    }
    char* wsb = static_cast<char*>(ws);
    const long long chunks = K / I::CH;
    uint32_t* epoch = reinterpret_cast<uint32_t*>(wsb + base);
    unsigned long long* tslots = reinterpret_cast<unsigned long long*>(wsb + base + 1024);
    const size_t frag_off = base + 1024 + kI8MaxWarps * kI8SlotBytes;
    uint8_t* frag = reinterpret_cast<uint8_t*>(wsb + frag_off);
    float2* terms = reinterpret_cast<float2*>(wsb + frag_off + (size_t)chunks * I::FRAG_CHUNK);

    const int W = p.warps_total < wpc ? p.warps_total : wpc;
    CUtensorMap wmap, smap, bmap;
    const uint64_t wrow = (uint64_t)K * BITS / 32;
    int rc = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, wrow, (uint64_t)N, wrow * 4, 32,
                           (uint32_t)R_::ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t G = (uint64_t)K / GS;
    const CUtensorMapDataType dt = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    rc = tensor_map_2d(&smap, dt, sc, G, (uint64_t)N, G * 2, 8, (uint32_t)R_::ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = tensor_map_2d(&bmap, dt, bi, G, (uint64_t)N, G * 2, 8, (uint32_t)R_::ROWS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;

    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t pcfg = {};
    pcfg.gridDim = dim3((unsigned)(K / GS), 1, 1);
    pcfg.blockDim = dim3(32, 1, 1);
    pcfg.stream = st;
    pcfg.attrs = attrs;
    pcfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&pcfg, prep, x, M, K, (int)(((uintptr_t)x & 15u) == 0), frag, terms, epoch);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_status(e, "qmv_i8 prep launch");
    }
    qmm::I8Args a{};
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.Ut = p.Ut;
    a.T = p.T;
    a.warps_total = p.warps_total;
    a.tslots = tslots;
    a.epoch = epoch;
    a.frag = frag;
    a.terms = terms;
    a.amax = amax;
    a.n_offset = n_offset;
    cudaLaunchConfig_t cfg = {};
    // warps past warps_total (a last CTA of fewer) find no unit and exit
    cfg.gridDim = dim3((unsigned)((p.warps_total + W - 1) / W), 1, 1);
    cfg.blockDim = dim3(32 * W, 1, 1);
    cfg.dynamicSmemBytes = smem_for(W);
    cfg.stream = st;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, wmap, smap, bmap, a);
    if (e != cudaSuccess) cudaGetLastError();
    return cuda_status(e, "qmv_i8 launch");
}

template <int BITS, int GS, bool F16>
static int launch_i8_m(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                       int M, int N, int K, void* ws, size_t ws_bytes, cudaStream_t st, unsigned long long* amax,
                       long long n_offset) {
    // Ring depth per warp: 2 stages on matrices under 128 MiB of codes, 4 above
    // (the lm_head class).  Measured on B200 (graphs of 20 launches): the
    // 248320x5120 8-bit lm_head takes 216 / 221 / 223 us at M = 1 / 4 / 8 with
    // 4 stages (8 warps per SM) against 230 / 227 / 279 us with 2 (16 warps per
    // SM); 17408x5120 takes 13.2 / 13.8 us at M = 1 / 4 with 2 stages against
    // 14.9 / 15.1 with 4.  The choice depends on the matrix only, so every
    // M <= 8 call on one matrix keeps one unit split (and single-row bits).
    if ((long long)N * K * BITS / 8 >= (128LL << 20)) {
        switch (i8_mp(M)) {
            case 1: return launch_i8_t<BITS, GS, F16, 1, 4>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
            case 4: return launch_i8_t<BITS, GS, F16, 4, 4>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
            default: return launch_i8_t<BITS, GS, F16, 8, 4>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
        }
    }
    switch (i8_mp(M)) {
        case 1: return launch_i8_t<BITS, GS, F16, 1, 2>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
        case 4: return launch_i8_t<BITS, GS, F16, 4, 2>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
        default: return launch_i8_t<BITS, GS, F16, 8, 2>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
    }
}

// Dense decode on warp-level integer MMA.  ws: qmm_quantized_matmul's
// workspace (its counter block zero).  amax (optional, zeroed by the caller):
// the fused greedy-sampling keys of the M rows, over global indices
// n_offset + n.
int launch_qmv_i8(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st,
                  unsigned long long* amax, long long n_offset) {
#define QMM_I8_CASE(B, S)                                                                                   \
    if (bits == B && gs == S)                                                                                \
        return f16 ? launch_i8_m<B, S, true>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset)     \
                   : launch_i8_m<B, S, false>(x, w, sc, bi, y, M, N, K, ws, ws_bytes, st, amax, n_offset);
    QMM_I8_CASE(4, 32)
    QMM_I8_CASE(4, 64)
    QMM_I8_CASE(4, 128)
    QMM_I8_CASE(8, 32)
    QMM_I8_CASE(8, 64)
    QMM_I8_CASE(8, 128)
#undef QMM_I8_CASE
    set_error("qmv_i8: bits=%d group_size=%d not supported", bits, gs);
    return QMM_EUNSUPPORTED;
}

size_t i8_total_workspace(long long M, long long N, long long K, int gs, int bits) {
    return i8_sk_part(M, N, K, gs, bits) + i8_extra_workspace(M, K, gs, bits);
}

int qmv_i8_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, qmm::g_i8_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(qmm::g_i8_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace qmm_host
