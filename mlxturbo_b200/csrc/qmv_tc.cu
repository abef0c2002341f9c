// qmv_tc.cu -- decode quantized matmul on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a, for few activation rows (M <= 8).
//
// Replaces the reference's decode GEMV path (mlxturbo/kernels/qmv_small_m.py:
// 79-218, qmv_wide_nocap.py, the MLX qmv kernel) where it is dispatched:
// y[m, n] = sum_k x[m, k] * (s[n, g] * q[n, k] + b[n, g]).
//
// Integer tensor-core formulation (tcgen05.mma kind::i8, exact s32 sums):
//
//   A = the codes q as u8 (128 weight rows x one stage of K).  4-bit codes
//       are expanded to bytes in TMEM, three integer ops per 8 weights
//       (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F: word w's logical K order is
//       q0 q2 q4 q6 q1 q3 q5 q7); 8-bit codes need no work at all: the TMA'd
//       weight tile (128-byte rows, 128-byte swizzle) is the A operand in
//       shared memory as it lands.
//   B = the activations as two exact int8 planes per quantisation group:
//       with e the largest f32 exponent of x over the group (one row),
//       X_k = rint(x_k * 2^(140 - e)) = 128 * d1_k + d0_k, |X_k| < 2^14,
//       d1 in s8, d0 in [0, 127].  Every value within 2^6 of the group's
//       largest is exact (bf16 / fp16 significands fit in 14 bits); smaller
//       ones are rounded to 2^(e - 141) absolute.  B is block diagonal:
//       row (g * MP + m) * 2 + p holds plane p of activation row m inside
//       group g's K range, zeros elsewhere, so one MMA chain yields every
//       (group, row, plane) partial sum D = sum_{k in g} q_k * d_p,k.
//   Epilogue, per stage and weight row (one TMEM lane per thread):
//       res[m] += s_g * 2^(e - 140) * (128 * D1 + D0) + b_g * sum_{k in g} x_k.
//
// The B tiles depend only on x and the K stage, so a small prep kernel
// (one warp per stage) builds every stage's tile and per-group terms once
// into the workspace; the main kernel copies a stage's tile into its ring
// slot beside the weights with one bulk copy on the same barrier.
//
// Schedule: one CTA per SM, stream-K over (128-row tile, K stage) units as
// in qmv_sk.cu (contiguous equal unit ranges per CTA; a tile cut between
// CTAs is summed through two partial slots per CTA by whichever CTA
// finishes it last, in CTA order, so results do not depend on timing).
// A stage is 128 packed bytes per weight row (256 values at 4 bits, 128 at 8).
//
// Warp roles:
//   0        TMA producer: weights (128 rows x 128 B, SW128) and the stage's
//            B tile into an S-deep ring;
//   1        MMA issuer (warp-uniform loop, one elected lane issues):
//            tcgen05.mma kind::i8, 128 x NB x 32 per instruction;
//   2..5     4-bit only: code expanders, one per TMEM lane quarter, into a
//            double-buffered TMEM A;
//   last 8   epilogue, two sets of four (even / odd stages of the CTA's
//            range), one warp per lane quarter: TMEM D (double-buffered) ->
//            per-group scaling (scales, biases and per-group terms loaded
//            from global memory stages ahead) -> running sums -> y or the
//            partial slots.
// Every mbarrier wait is bounded; a wait that gives up sets the device error
// flag and the kernel drains (no new loads, outstanding loads and MMAs
// waited for, TMEM freed).

#include <stdlib.h>

#include "tc.cuh"
#include "tma.cuh"

namespace qmm {

__device__ int g_tc_error;

constexpr int tc_pow2_cols(int c) { return c <= 32 ? 32 : c <= 64 ? 64 : c <= 128 ? 128 : c <= 256 ? 256 : 512; }

template <int BITS, int GS, bool F16, int MP>
struct TcCfg {
    static constexpr int ROWS = 128;                  // weight rows per tile (MMA M)
    static constexpr int WB = 128;                    // packed bytes per row per stage
    static constexpr int RK = WB * 8 / BITS;          // K per stage (256 or 128)
    static constexpr int KI = RK / 32;                // MMAs per stage (K = 32 bytes each)
    static constexpr int RPC = 32 / BITS;             // activation values per prep lane and row (8 or 4)
    static constexpr int LPG = GS / RPC;              // prep lanes per group
    static constexpr int GPS = RK / GS;               // groups per stage
    static constexpr int NPAIR = GPS * MP;            // (group, row) pairs per stage
    static constexpr int ND = 2 * NPAIR;              // used D columns: (group, row, plane)
    static constexpr int NB = ND < 16 ? 16 : (ND + 15) / 16 * 16;  // MMA N
    static_assert(RK % GS == 0 && LPG >= 1 && LPG <= 32, "group geometry");
    static_assert(RK / RPC == 32 && GPS * LPG == 32, "one prep lane per RPC activation values of a stage");
    static_assert(ND <= 64, "D columns per stage (registers of the epilogue)");
    static constexpr bool A_TMEM = BITS == 4;         // 8-bit codes are the A operand in shared memory
    static constexpr int A_COLS = A_TMEM ? RK / 4 : 0;  // TMEM columns per A stage (4 bytes of K each)
    // TMEM rings: A (4-bit codes as bytes) and D (accumulators), each as
    // deep as the 512 columns allow, up to 4 (a 2-deep ring makes the
    // expander -> MMA -> expander and MMA -> epilogue -> MMA hand-offs
    // two-stage cycles whose barrier latency sets the pace)
    static constexpr int NAB = A_TMEM ? 4 : 1;       // A buffers
    static constexpr int NDB = (NAB * A_COLS + 4 * NB <= 512) ? 4 : 2;  // D buffers (even: two per epilogue set)
    static constexpr int D_COL = NAB * A_COLS;
    static constexpr int TMEM_COLS = tc_pow2_cols(D_COL + NDB * NB);
    static_assert(D_COL + NDB * NB <= 512, "TMEM budget");
    static constexpr int DQW = A_TMEM ? 4 : 0;        // code-expander warps, one per TMEM lane quarter
    static constexpr int EPI0 = 2 + DQW;              // first epilogue warp
    static constexpr int EPW = 8;                     // epilogue warps: two sets of four (even / odd stages)
    static constexpr int THREADS = 32 * (EPI0 + EPW);
    // B tile of one stage: RK / 128 SW128 sub-tiles of NB rows x 128 bytes (128 K)
    static constexpr int BSUBS = RK / 128;
    static constexpr int B_SUB = NB * 128;
    static constexpr int B_BYTES = BSUBS * B_SUB;
    // prep output per stage: the B tile, then (sum of x, 2^(e-140)) per (group, row)
    static constexpr int PREP_STRIDE = (B_BYTES + NPAIR * 8 + 127) / 128 * 128;
    // ring slot: weights | B tile
    static constexpr int W_BYTES = ROWS * WB;         // 16 KiB
    static constexpr int B_OFF = W_BYTES;
    static constexpr int SLOT = (W_BYTES + B_BYTES + 1023) / 1024 * 1024;
    // Shared memory is held to 200 KB: with allocations near the 227 KB
    // maximum an earlier layout of this kernel returned wrong rows
    // (timing-dependent); the limit stays well below.
    static constexpr int SMEM_MAX = 204800;
    static constexpr int CMB_BYTES = ROWS * MP * 4;   // odd set's partial sums at a tile end
    static constexpr int FIXED = CMB_BYTES + 512 + 1024;
    static constexpr int S_FIT = (SMEM_MAX - FIXED) / SLOT;
    static constexpr int S = S_FIT > 12 ? 12 : S_FIT;  // weight ring depth (bytes in flight per SM)
    static_assert(S >= 3, "ring too shallow");
    static constexpr int CMB_OFF = S * SLOT;
    static constexpr int BAR_OFF = CMB_OFF + CMB_BYTES;
    static constexpr int NBARS = 2 * S + 2 * NAB + 2 * NDB + 1;
    static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
    static constexpr int TOTAL = MISC_OFF + 16 + 1024;  // + alignment slack
    static_assert(TOTAL <= SMEM_MAX, "shared memory budget");
};

struct TcArgs {
    const uint16_t* sc;   // scales / biases [N][K / GS], read by the epilogue directly
    const uint16_t* bi;
    const uint8_t* prep;  // [Ut][PREP_STRIDE]: B tile and per-group terms of each K stage
    uint16_t* y;
    int M, N, K;
    int Ut;               // K stages per tile
    int T;                // row tiles
    float* slots;         // [ctas][2][MP][128]
    int* counters;        // [T], zero between calls
};

// Bounded wait on an mbarrier phase.  A non-suspending test first (a phase
// that already completed costs one barrier access), then polls that may
// suspend the warp for up to 200 ns each.  About 2^20 polls before it gives up.
QMM_DEVINL bool tc_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    for (uint32_t i = 0; i < (1u << 20); ++i) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity), "r"(200u)
            : "memory");
        if (ok) return true;
        if (*abort) return false;
    }
    *abort = 1;
    atomicExch(&g_tc_error, 1);
    return false;
}

// Bounded wait that ignores the abort flag: used while draining, for copies
// and MMAs that were issued and always complete.
QMM_DEVINL void tc_wait_final(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return;
    }
    atomicExch(&g_tc_error, 1);
}

QMM_DEVINL void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

QMM_DEVINL int tc_atom_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

QMM_DEVINL int tc_owner(long long u, long long total, int wt) { return (int)(((u + 1) * wt - 1) / total); }

template <int N_>
QMM_DEVINL void tmem_ld_cols(uint32_t taddr, uint32_t (&v)[N_]) {
    if constexpr (N_ == 1) tmem_ld1(taddr, v);
    else if constexpr (N_ == 2) tmem_ld2(taddr, v);
    else if constexpr (N_ == 4) tmem_ld4(taddr, v);
    else if constexpr (N_ == 8) tmem_ld8(taddr, v);
    else if constexpr (N_ == 16) tmem_ld16(taddr, v);
    else {
        static_assert(N_ % 32 == 0, "column count");
#pragma unroll
        for (int c = 0; c < N_; c += 32) tmem_ld32(taddr + c, *reinterpret_cast<uint32_t(*)[32]>(&v[c]));
    }
}

// Exact conversion of an integer below 2^22 in magnitude to f32: add it to
// the bit pattern of 1.5 * 2^23 and subtract that value again.
QMM_DEVINL float small_int_to_f32(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }

// GPS consecutive 16-bit scales (or biases) of one weight row, loaded as one vector.
template <int GPS>
struct ScaleVec {
    uint32_t w[(GPS + 1) / 2];
};
template <int GPS>
QMM_DEVINL ScaleVec<GPS> load_scales(const uint16_t* p) {
    ScaleVec<GPS> v;
    if constexpr (GPS == 8) {
        const uint4 q = ldg_stream_v4(p);
        v.w[0] = q.x;
        v.w[1] = q.y;
        v.w[2] = q.z;
        v.w[3] = q.w;
    } else if constexpr (GPS == 4) {
        const uint2 q = ldg_stream_v2(p);
        v.w[0] = q.x;
        v.w[1] = q.y;
    } else if constexpr (GPS == 2) {
        v.w[0] = ldg_stream_u32(p);
    } else {
        v.w[0] = ldg_u16(p);
    }
    return v;
}
template <bool F16, int GPS>
QMM_DEVINL float scale_at(const ScaleVec<GPS>& v, int g) {
    return (g & 1) ? Half<F16>::hi_f32(v.w[g >> 1]) : Half<F16>::lo_f32(v.w[g >> 1]);
}

// Int8 activation planes of one K stage (MP rows) in the B-tile layout the
// main kernel's MMAs read (block diagonal, SW128 K-major), and the per-group
// terms.  One warp per stage; lane j takes RPC values of each row.
template <int BITS, int GS, bool F16, int MP>
__global__ void __launch_bounds__(32) qmv_tc_prep_kernel(const uint16_t* __restrict__ x, int M, int K,
                                                         uint8_t* __restrict__ prep) {
    using C = TcCfg<BITS, GS, F16, MP>;
    using H = Half<F16>;
    constexpr int XW = C::RPC / 2;  // 32-bit words of x per lane and row
    pdl_launch_dependents();
    pdl_wait();  // x is the previous kernel's output
    const int ku = blockIdx.x, j = threadIdx.x, g = j / C::LPG;
    uint8_t* tile = prep + (size_t)ku * C::PREP_STRIDE;
    float2* sxr = reinterpret_cast<float2*>(tile + C::B_BYTES);
    for (int q = j; q < C::B_BYTES / 16; q += 32) reinterpret_cast<uint4*>(tile)[q] = make_uint4(0, 0, 0, 0);
    uint32_t v[MP][XW];
#pragma unroll
    for (int m = 0; m < MP; ++m) {
        if (m < M) {
            const uint16_t* xp = x + (size_t)m * K + (size_t)ku * C::RK + C::RPC * j;
            if constexpr (XW == 4) {
                const uint4 q = ldg_v4(xp);
                v[m][0] = q.x;
                v[m][1] = q.y;
                v[m][2] = q.z;
                v[m][3] = q.w;
            } else {
                const uint2 q = *reinterpret_cast<const uint2*>(xp);
                v[m][0] = q.x;
                v[m][1] = q.y;
            }
        }
    }
    __syncwarp();  // the zeros are written before the diagonal blocks
#pragma unroll
    for (int m = 0; m < MP; ++m) {
        if (m >= M) {
            if ((j & (C::LPG - 1)) == 0) sxr[g * MP + m] = make_float2(0.0f, 0.0f);
            continue;  // warp-uniform
        }
        float f[C::RPC];
#pragma unroll
        for (int e = 0; e < XW; ++e) {
            f[2 * e] = H::lo_f32(v[m][e]);
            f[2 * e + 1] = H::hi_f32(v[m][e]);
        }
        float amax = 0.0f, sum = 0.0f;
#pragma unroll
        for (int e = 0; e < C::RPC; ++e) {
            amax = fmaxf(amax, fabsf(f[e]));
            sum += f[e];
        }
#pragma unroll
        for (int off = C::LPG / 2; off >= 1; off >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            sum += __shfl_xor_sync(0xffffffffu, sum, off);
        }
        // group exponent (f32 bias); tiny or zero groups use the smallest scale
        int e = (int)((__float_as_uint(amax) >> 23) & 0xFFu);
        e = e < 14 ? 14 : e;
        const float up = __uint_as_float((uint32_t)(267 - e) << 23);  // 2^(140 - e)
        // X = rint(x * 2^(140-e)) rides in the low bits of 1.5 * 2^23 + X:
        // bits 0..6 are d0, bits 7..14 the s8 pattern of d1
        uint32_t bx[C::RPC];
#pragma unroll
        for (int e2 = 0; e2 < C::RPC; ++e2) bx[e2] = __float_as_uint(fmaf(f[e2], up, 12582912.0f));
        // plane bytes in the A operand's K order: 4-bit words run
        // q0 q2 q4 q6 | q1 q3 q5 q7, 8-bit words are in natural order
        uint32_t p0[C::RPC / 4], p1[C::RPC / 4];
#pragma unroll
        for (int h = 0; h < C::RPC / 4; ++h) {
            const int i0 = C::RPC == 8 ? h : 4 * h;  // first value of this 4-byte word
            const int st = C::RPC == 8 ? 2 : 1;      // value stride inside it
            const uint32_t lo = prmt(bx[i0], bx[i0 + st], 0x5410);
            const uint32_t hi = prmt(bx[i0 + 2 * st], bx[i0 + 3 * st], 0x5410);
            p0[h] = prmt(lo, hi, 0x6420) & 0x7F7F7F7Fu;
            p1[h] = prmt(lo >> 7, hi >> 7, 0x6420);
        }
        const int r0 = (g * MP + m) * 2;  // plane 0 row; plane 1 is r0 + 1
        constexpr int LB = C::RPC;        // bytes per plane per lane
        const int L = LB * j;             // logical K byte of this lane in the stage
        uint8_t* sub = tile + (L >> 7) * C::B_SUB;
        const int w16 = (L & 127) >> 4, o16 = L & 15;
        uint8_t* d0p = sub + r0 * 128 + ((w16 ^ (r0 & 7)) << 4) + o16;
        uint8_t* d1p = sub + (r0 + 1) * 128 + ((w16 ^ ((r0 + 1) & 7)) << 4) + o16;
        if constexpr (LB == 8) {
            *reinterpret_cast<uint2*>(d0p) = make_uint2(p0[0], p0[1]);
            *reinterpret_cast<uint2*>(d1p) = make_uint2(p1[0], p1[1]);
        } else {
            *reinterpret_cast<uint32_t*>(d0p) = p0[0];
            *reinterpret_cast<uint32_t*>(d1p) = p1[0];
        }
        if ((j & (C::LPG - 1)) == 0) sxr[g * MP + m] = make_float2(sum, __uint_as_float((uint32_t)(e - 13) << 23));
    }
}

template <int BITS, int GS, bool F16, int MP>
__global__ void __launch_bounds__(TcCfg<BITS, GS, F16, MP>::THREADS, 1)
    qmv_tc_kernel(const __grid_constant__ CUtensorMap wmap, TcArgs a) {
    using C = TcCfg<BITS, GS, F16, MP>;
    using H = Half<F16>;
    constexpr int S = C::S, GPS = C::GPS, ND = C::ND, NPAIR = C::NPAIR;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + C::BAR_OFF;
    auto full = [&](int s) { return bar0 + 8 * s; };
    auto empty = [&](int s) { return bar0 + 8 * (S + s); };
    constexpr int NAB = C::NAB, NDB = C::NDB;
    auto afull = [&](int b) { return bar0 + 8 * (2 * S + b); };
    auto aempty = [&](int b) { return bar0 + 8 * (2 * S + NAB + b); };
    auto dfull = [&](int b) { return bar0 + 8 * (2 * S + 2 * NAB + b); };
    auto dempty = [&](int b) { return bar0 + 8 * (2 * S + 2 * NAB + NDB + b); };
    const uint32_t mdone = bar0 + 8 * (2 * S + 2 * NAB + 2 * NDB);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::MISC_OFF);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 4);
    volatile int* sh_prev = reinterpret_cast<volatile int*>(smem + C::MISC_OFF + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long total = (long long)a.T * a.Ut;
    const int wt = gridDim.x, gw = blockIdx.x;
    const long long ua = total * gw / wt, ub = total * (gw + 1) / wt;
    const int nst = (int)(ub - ua);

    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), C::DQW + 1);  // code expanders, MMA commit (B tile; 8-bit: also the codes)
        }
        for (int b = 0; b < NAB; ++b) {
            mbar_init(afull(b), C::DQW > 0 ? C::DQW : 1);
            mbar_init(aempty(b), 1);
        }
        for (int b = 0; b < NDB; ++b) {
            mbar_init(dfull(b), 1);
            mbar_init(dempty(b), 4);
        }
        mbar_init(mdone, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer (warp-uniform loop, one elected lane issues) ----------------
        if (nst > 0) {
            if (elect_one()) tma_prefetch_desc(&wmap);
            constexpr uint32_t tx = C::W_BYTES + C::B_BYTES;
            int tile = (int)(ua / a.Ut), ku = (int)(ua - (long long)tile * a.Ut);
            // weights of the next stage into slot s; returns the stage's K index
            auto issue_w = [&](int s) {
                const uint32_t dst = sbase + s * C::SLOT;
                const int wrow = tile * C::ROWS, kw = ku * (C::WB / 4);
                if (elect_one()) {
                    mbar_expect_tx(full(s), tx);
                    tma_load_2d(dst, &wmap, full(s), kw, wrow);
                }
                __syncwarp();
                const int k = ku;
                if (++ku == a.Ut) {
                    ku = 0;
                    ++tile;
                }
                return k;
            };
            // the stage's B tile, built by the prep kernel
            auto issue_b = [&](int s, int k) {
                if (elect_one())
                    bulk_load(sbase + s * C::SLOT + C::B_OFF, a.prep + (size_t)k * C::PREP_STRIDE, C::B_BYTES, full(s));
                __syncwarp();
            };
            // the weights do not depend on the previous kernels: stream them first
            const int pre = nst < S ? nst : S;
            const int ku0 = ku;
            for (int i = 0; i < pre; ++i) issue_w(i);
            pdl_wait();
            {
                int k = ku0;
                for (int i = 0; i < pre; ++i) {
                    issue_b(i, k);
                    if (++k == a.Ut) k = 0;
                }
            }
            int issued = pre;
            for (int i = pre; i < nst; ++i) {
                const int s = i % S;
                if (!tc_wait(empty(s), ((uint32_t)(i / S) & 1u) ^ 1u, abort)) break;
                const int k = issue_w(s);
                issue_b(s, k);
                issued = i + 1;
            }
            // drain: every issued copy has landed before the CTA exits
            for (int i = issued - S < 0 ? 0 : issued - S; i < issued; ++i)
                tc_wait_final(full(i % S), (uint32_t)(i / S) & 1u);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (warp-uniform loop, one elected lane issues) ----------------
        constexpr uint32_t idesc = umma_idesc_i8(128, C::NB);
        int s = 0;
        for (int i = 0; i < nst; ++i) {
            const int ab = i % NAB, db = i % NDB;
            tc_wait(full(s), (uint32_t)(i / S) & 1u, abort);  // the stage's B tile (8-bit: and the codes)
            if constexpr (C::A_TMEM) tc_wait(afull(ab), (uint32_t)(i / NAB) & 1u, abort);
            tc_wait(dempty(db), ((uint32_t)(i / NDB) & 1u) ^ 1u, abort);
            tc_fence_after();
            const uint32_t d_col = tmem + (uint32_t)(C::D_COL + db * C::NB);
            const uint64_t bdesc = umma_desc_sw128(sbase + s * C::SLOT + C::B_OFF);
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < C::KI; ++kk) {
                    // B: sub-tile kk / 4, 32-byte K step inside it (>> 4 in the address field)
                    const uint64_t bd = bdesc + (uint64_t)(((kk >> 2) * C::B_SUB + (kk & 3) * 32) >> 4);
                    if constexpr (C::A_TMEM)
                        umma_i8_ts(d_col, tmem + (uint32_t)(ab * C::A_COLS + 8 * kk), bd, idesc, kk != 0);
                    else
                        umma_i8(d_col, umma_desc_sw128(sbase + s * C::SLOT + 32 * kk), bd, idesc, kk != 0);
                }
                if constexpr (C::A_TMEM) umma_commit(aempty(ab));
                umma_commit(empty(s));  // the slot's B tile (and 8-bit codes) were read
                umma_commit(dfull(db));
            }
            __syncwarp();
            if (++s == S) s = 0;
        }
        if (elect_one()) umma_commit(mdone);
        __syncwarp();
        tc_wait_final(mdone, 0);
    } else if (warp < C::EPI0) {
        // ---------------- 4-bit code expanders: one per TMEM lane quarter ----------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        for (int i = 0; i < nst; ++i) {
            const int s = i % S, ab = i % NAB;
            tc_wait(full(s), (uint32_t)(i / S) & 1u, abort);
            const uint8_t* wrow = smem + s * C::SLOT + row * 128;
            uint32_t wv[32];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 pk = *reinterpret_cast<const uint4*>(wrow + ((c ^ (row & 7)) << 4));
                wv[4 * c] = pk.x;
                wv[4 * c + 1] = pk.y;
                wv[4 * c + 2] = pk.z;
                wv[4 * c + 3] = pk.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty(s));
            tc_wait(aempty(ab), ((uint32_t)(i / NAB) & 1u) ^ 1u, abort);
            tc_fence_after();
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                uint32_t av[32];
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) {
                    av[2 * jj] = wv[16 * hh + jj] & 0x0F0F0F0Fu;             // q0 q2 q4 q6
                    av[2 * jj + 1] = (wv[16 * hh + jj] >> 4) & 0x0F0F0F0Fu;  // q1 q3 q5 q7
                }
                tmem_st32(t_lane + (uint32_t)(ab * C::A_COLS + 32 * hh), av);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(afull(ab));
        }
    } else {
        // ---------------- epilogue: set 0 takes the even stages of the range, set 1 the odd ----------------
        pdl_wait();  // y, the slots, the counters and the prep output belong to earlier kernels
        const int set = (warp - C::EPI0) >> 2, quarter = warp & 3, et = (warp - C::EPI0 - 4 * set) * 32 + lane;
        const int row = quarter * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        const int G = a.K / GS;
        float* cmb = reinterpret_cast<float*>(smem + C::CMB_OFF);
        float res[MP];
#pragma unroll
        for (int m = 0; m < MP; ++m) res[m] = 0.0f;

        // scales and biases of unit ua + i for this thread's weight row, two
        // of this set's stages ahead (rows past N read row N - 1; dropped later)
        auto fetch = [&](int i, ScaleVec<GPS>& sv, ScaleVec<GPS>& bv) {
            if (i < nst) {
                const int u = (int)(ua + i), t = u / a.Ut, k = u - t * a.Ut;
                int n = t * C::ROWS + row;
                n = n < a.N ? n : a.N - 1;
                const long long off = (long long)n * G + k * GPS;
                sv = load_scales<GPS>(a.sc + off);
                bv = load_scales<GPS>(a.bi + off);
            }
        };
        ScaleVec<GPS> s0{}, b0{}, s1{}, b1{}, s2{}, b2{};
        fetch(set, s0, b0);
        fetch(set + 2, s1, b1);
        fetch(set + 4, s2, b2);

        int tile = (int)(ua / a.Ut), ku = (int)(ua - (long long)tile * a.Ut), k0 = ku;
        auto flush = [&](int t, int kb, int ke) {
            // the odd set's partial sums join the even set's
            if (set == 1) {
#pragma unroll
                for (int m = 0; m < MP; ++m) cmb[m * C::ROWS + row] = res[m];
            }
            named_sync(1, 256);
            if (set == 0) {
#pragma unroll
                for (int m = 0; m < MP; ++m) res[m] += cmb[m * C::ROWS + row];
            }
            named_sync(1, 256);  // the odd set overwrites cmb only after this
            if (set == 1) return;
            const int n = t * C::ROWS + row;
            float out[MP];
            bool store = (kb == 0 && ke == a.Ut);
            if (store) {
#pragma unroll
                for (int m = 0; m < MP; ++m) out[m] = res[m];
            } else {
                const long long u0 = (long long)t * a.Ut;
                const int f = tc_owner(u0, total, wt), l = tc_owner(u0 + a.Ut - 1, total, wt);
                // a CTA's slot 1 holds the tile its range ends in when that
                // range started before the tile; every other partial uses slot 0
                const bool f_before = total * f / wt < u0;
                auto slot_of = [&](int w) {
                    return a.slots + ((long long)w * 2 + (w == f && f_before ? 1 : 0)) * (MP * C::ROWS) + row;
                };
                float* mine = slot_of(gw);
#pragma unroll
                for (int m = 0; m < MP; ++m) mine[m * C::ROWS] = res[m];
                named_sync(2, 128);  // every even-set thread's slot stores precede the release
                if (et == 0) *sh_prev = tc_atom_add_acq_rel(a.counters + t, 1);
                named_sync(2, 128);
                if (*sh_prev == l - f) {
#pragma unroll
                    for (int m = 0; m < MP; ++m) out[m] = 0.0f;
                    for (int w = f; w <= l; ++w) {
                        const float* p = slot_of(w);
#pragma unroll
                        for (int m = 0; m < MP; ++m) out[m] += __ldcg(p + m * C::ROWS);
                    }
                    if (et == 0) a.counters[t] = 0;
                    store = true;
                }
            }
            if (store && n < a.N) {
#pragma unroll
                for (int m = 0; m < MP; ++m)
                    if (m < a.M) a.y[(long long)m * a.N + n] = H::from_f32(out[m]);
            }
        };

        for (int i = 0; i < nst; ++i) {
            if ((i & 1) == set) {
                const int db = i % NDB;
                // per-group terms of this stage (the same for every row), in
                // flight while the MMA result is awaited
                const float4* gp = reinterpret_cast<const float4*>(a.prep + (size_t)ku * C::PREP_STRIDE + C::B_BYTES);
                float4 gq[(NPAIR + 1) / 2];
#pragma unroll
                for (int c = 0; c < (NPAIR + 1) / 2; ++c) gq[c] = __ldg(gp + c);
                tc_wait(dfull(db), (uint32_t)(i / NDB) & 1u, abort);
                tc_fence_after();
                uint32_t d[ND];
                tmem_ld_cols<ND>(t_lane + (uint32_t)(C::D_COL + db * C::NB), d);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(dempty(db));
#pragma unroll
                for (int g = 0; g < GPS; ++g) {
                    const float sf = scale_at<F16, GPS>(s0, g), bf = scale_at<F16, GPS>(b0, g);
#pragma unroll
                    for (int m = 0; m < MP; ++m) {
                        const int c = g * MP + m;
                        const float gsum = (c & 1) ? gq[c >> 1].z : gq[c >> 1].x;  // sum of x over the group
                        const float gsc = (c & 1) ? gq[c >> 1].w : gq[c >> 1].y;   // 2^(e - 140)
                        const float dq =
                            fmaf(small_int_to_f32((int)d[2 * c + 1]), 128.0f, small_int_to_f32((int)d[2 * c]));
                        res[m] = fmaf(sf * gsc, dq, res[m]);
                        res[m] = fmaf(bf, gsum, res[m]);
                    }
                }
                s0 = s1;
                b0 = b1;
                s1 = s2;
                b1 = b2;
                fetch(i + 6, s2, b2);
            }
            const bool last = (i == nst - 1);
            if (++ku == a.Ut || last) {
                flush(tile, k0, ku);
#pragma unroll
                for (int m = 0; m < MP; ++m) res[m] = 0.0f;
                if (ku == a.Ut) {
                    ku = 0;
                    ++tile;
                }
                k0 = ku;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS)
                     : "memory");
    }
}

}  // namespace qmm

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace qmm_host {

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) !=
                                                      cudaSuccess)
            n = 148;
    }
    return n;
}

// QMM_TC_CTAS overrides the CTA count (tuning).
static int env_int(const char* name, int dflt) {
    const char* e = getenv(name);
    return (e && *e) ? atoi(e) : dflt;
}

static int tc_mp(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8; }

// Whether the tensor-core decode kernel supports this problem.
size_t tc_workspace(int M, long long K, int gs, int bits);

bool tc_eligible(int M, long long N, long long K, int gs, int bits, bool f16, const void* x, const void* sc,
                 const void* bi) {
    (void)f16;
    if (M < 1 || M > 8) return false;
    if (bits != 4 && bits != 8) return false;
    if (gs != 32 && gs != 64 && gs != 128) return false;
    const int rk = 128 * 8 / bits;
    if (K % rk != 0 || (K / gs) % 8 != 0) return false;      // whole stages; 16-byte scale rows
    if (bits == 4 && gs == 32 && M > 4) return false;       // 8 groups x 8 rows x 2 planes > 64 D columns
    if (((uintptr_t)x | (uintptr_t)sc | (uintptr_t)bi) & 15u) return false;
    if ((N + 127) / 128 > 65536) return false;
    // its scratch stays below the 8 MiB where the integer-MMA kernel's begins
    if (tc_workspace(M, K, gs, bits) > (8u << 20)) return false;
    return true;
}

// Bytes per K stage of the prep output (the same formula as TcCfg::PREP_STRIDE).
static constexpr size_t tc_prep_stride(int bits, int gs, int mp) {
    const int rk = 1024 / bits, npair = rk / gs * mp, nd = 2 * npair;
    const int nb = nd < 16 ? 16 : (nd + 15) / 16 * 16;
    return ((size_t)(rk / 128) * nb * 128 + (size_t)npair * 8 + 127) / 128 * 128;
}

// Workspace: 256 KiB of tile counters (zero between calls), two partial
// slots per CTA, then the prep output of every K stage.
static size_t tc_prep_offset(int M) {
    return ((size_t)65536 * sizeof(int) + (size_t)sm_count() * 2 * 128 * tc_mp(M) * sizeof(float) + 1023) / 1024 * 1024;
}
size_t tc_workspace(int M, long long K, int gs, int bits) {
    if (bits != 4 && bits != 8) return 0;
    return tc_prep_offset(M) + (size_t)(K / (1024 / bits)) * tc_prep_stride(bits, gs, tc_mp(M));
}

template <int BITS, int GS, bool F16, int MP>
static int launch_tc_t(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                       int M, int N, int K, void* ws, cudaStream_t st) {
    using C = qmm::TcCfg<BITS, GS, F16, MP>;
    static_assert(C::PREP_STRIDE == tc_prep_stride(BITS, GS, MP), "prep layout");
    auto kern = qmm::qmv_tc_kernel<BITS, GS, F16, MP>;
    auto prep = qmm::qmv_tc_prep_kernel<BITS, GS, F16, MP>;
    {
        const int rc0 = ensure_smem_limit((const void*)kern, C::TOTAL, "qmv_tc smem attribute");
        if (rc0) return rc0;
    }
    qmm::TcArgs a{};
    a.sc = sc;
    a.bi = bi;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.T = (N + C::ROWS - 1) / C::ROWS;
    a.Ut = K / C::RK;
    const long long total = (long long)a.T * a.Ut;
    long long ctas = env_int("QMM_TC_CTAS", sm_count());
    if (ctas < 1) ctas = 1;
    if (ctas > sm_count()) ctas = sm_count();
    if (ctas > total) ctas = total;
    char* wsb = static_cast<char*>(ws);
    a.counters = reinterpret_cast<int*>(wsb);
    a.slots = reinterpret_cast<float*>(wsb + (size_t)65536 * sizeof(int));
    uint8_t* prep_out = reinterpret_cast<uint8_t*>(wsb + tc_prep_offset(M));
    a.prep = prep_out;

    CUtensorMap wmap;
    const uint64_t wrow = (uint64_t)K * BITS / 32;
    int rc = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, wrow, (uint64_t)N, wrow * 4, C::WB / 4,
                           (uint32_t)C::ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;

    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    // the activation planes of every K stage (one warp each)
    cudaLaunchConfig_t pcfg = {};
    pcfg.gridDim = dim3((unsigned)a.Ut, 1, 1);
    pcfg.blockDim = dim3(32, 1, 1);
    pcfg.stream = st;
    pcfg.attrs = attrs;
    pcfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaError_t e = cudaLaunchKernelEx(&pcfg, prep, x, M, K, prep_out);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_status(e, "qmv_tc prep launch");
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctas, 1, 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::TOTAL;
    cfg.stream = st;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, kern, wmap, a);
    if (e != cudaSuccess) cudaGetLastError();
    return cuda_status(e, "qmv_tc launch");
}

template <int BITS, int GS, bool F16>
static int launch_tc_m(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                       int M, int N, int K, void* ws, cudaStream_t st) {
    switch (tc_mp(M)) {
        case 1: return launch_tc_t<BITS, GS, F16, 1>(x, w, sc, bi, y, M, N, K, ws, st);
        case 2: return launch_tc_t<BITS, GS, F16, 2>(x, w, sc, bi, y, M, N, K, ws, st);
        case 4: return launch_tc_t<BITS, GS, F16, 4>(x, w, sc, bi, y, M, N, K, ws, st);
        default:
            if constexpr (BITS == 4 && GS == 32) {
                set_error("qmv_tc: 4-bit group size 32 takes M <= 4");
                return QMM_EUNSUPPORTED;
            } else {
                return launch_tc_t<BITS, GS, F16, 8>(x, w, sc, bi, y, M, N, K, ws, st);
            }
    }
}

// Dense decode on the tensor cores.  ws: tc_workspace(M, K, gs, bits) bytes, its first
// 256 KiB (tile counters) zero.
int launch_qmv_tc(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st) {
    if (ws_bytes < tc_workspace(M, K, gs, bits)) {
        set_error("qmv_tc: workspace %zu < %zu bytes", ws_bytes, tc_workspace(M, K, gs, bits));
        return QMM_EINVAL;
    }
#define QMM_TC_CASE(B, S)                                                                               \
    if (bits == B && gs == S)                                                                            \
        return f16 ? launch_tc_m<B, S, true>(x, w, sc, bi, y, M, N, K, ws, st)                           \
                   : launch_tc_m<B, S, false>(x, w, sc, bi, y, M, N, K, ws, st);
    QMM_TC_CASE(4, 32)
    QMM_TC_CASE(4, 64)
    QMM_TC_CASE(4, 128)
    QMM_TC_CASE(8, 32)
    QMM_TC_CASE(8, 64)
    QMM_TC_CASE(8, 128)
#undef QMM_TC_CASE
    set_error("qmv_tc: bits=%d group_size=%d f16=%d not supported", bits, gs, (int)f16);
    return QMM_EUNSUPPORTED;
}

int qmv_tc_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, qmm::g_tc_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(qmm::g_tc_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace qmm_host
