// prefill.cu -- M > 16 quantized matmul on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a.
//
// Replaces the reference's prefill kernels: MLX dense qmm_t (restated in
// mlxturbo/kernels/qmm_wide.py:53-66 and _steel_flat.py qmm_t_impl) and the
// BM=64 qmm_wide variant (qmm_wide.py:106-275).  Same arithmetic as qmm_t:
// each weight is dequantised to T (= s*q + b rounded once to bf16/fp16) and
// the T x T products accumulate in fp32.
//
// One CTA computes a 128 (weight rows) x BT (tokens) tile of y^T:
//   warp 0      TMA producer: x tile [BT x 64] (SW128) and the packed weight
//               tile [128 rows x 64 values] into a STAGES-deep smem ring;
//   warp 1      allocates TMEM and issues tcgen05.mma (one thread) with A
//               read from TMEM: D[128 x BT] += A[128 x 16] * B[BT x 16]^T,
//               four per k-block;
//   warps 2..9  dequantise the packed tile straight into TMEM (the A
//               stages), two warps per TMEM lane quarter (one K half each),
//               then run the epilogue TMEM -> registers -> y.
// Weights are the A operand (M=128) so each dequantised tile feeds BT tokens.
// Every mbarrier wait is bounded; a wait that gives up sets a device error
// flag (qmm_device_error) and the kernel runs to completion.

#include <stdlib.h>

#include "tc.cuh"
#include "tma.cuh"

namespace qmm {

__device__ int g_dev_error;

constexpr int PF_BW = 128;  // weight rows per CTA (MMA M)
constexpr int PF_BK = 64;   // K per stage

// Bounded wait recording failures in this file's error flag.
// Bounded wait recording failures in this file's error flag.  A
// non-suspending test first and between polls: a plain try_wait that finds
// the phase incomplete may suspend the thread for an implementation-defined
// time, well past the phase's completion; polls here suspend for at most a
// 20 ns hint.  About 2^22 polls before it gives up.
QMM_DEVINL bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    for (uint32_t i = 0; i < (1u << 22); ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 255u) == 255u && *abort) return false;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity), "r"(20u)
            : "memory");
        if (ok) return true;
    }
    *abort = 1;
    atomicExch(&g_dev_error, 1);
    return false;
}

template <bool F16, int BT>
struct PfIdesc {
    // D f32, A/B bf16 (1) or f16 (0), both K-major, N = BT, M = 128.
    static constexpr uint32_t value = (1u << 4) | ((F16 ? 0u : 1u) << 7) | ((F16 ? 0u : 1u) << 10) |
                                      ((uint32_t)(BT >> 3) << 17) | ((uint32_t)(PF_BW >> 4) << 24);
};

// Two packed pairs -> natural order: (lo.x, hi.x) and (lo.y, hi.y).
QMM_DEVINL uint32_t pair_lo(uint32_t a, uint32_t b) { return prmt(a, b, 0x5410); }
QMM_DEVINL uint32_t pair_hi(uint32_t a, uint32_t b) { return prmt(a, b, 0x7632); }

template <bool F16>
QMM_DEVINL uint32_t fma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    if constexpr (F16) asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    else asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Eight 4-bit codes of one word -> eight T values s*q+b in natural K order.
template <bool F16>
QMM_DEVINL uint4 deq8_4bit(uint32_t w, uint32_t s2, uint32_t b2) {
    using H = Half<F16>;
    constexpr uint32_t MASK = 0x000F000Fu;
    const uint32_t one2 = H::kOne2;
    const uint32_t neg_off2 = F16 ? 0xE400E400u : 0xC300C300u;  // (-1024, -1024) / (-128, -128)
    uint32_t p04 = fma2<F16>(and_or(w, MASK, H::kMagic), one2, neg_off2);        // (q0, q4)
    uint32_t p15 = fma2<F16>(and_or(w >> 4, MASK, H::kMagic), one2, neg_off2);   // (q1, q5)
    uint32_t p26 = fma2<F16>(and_or(w >> 8, MASK, H::kMagic), one2, neg_off2);   // (q2, q6)
    uint32_t p37 = fma2<F16>(and_or(w >> 12, MASK, H::kMagic), one2, neg_off2);  // (q3, q7)
    p04 = fma2<F16>(p04, s2, b2);
    p15 = fma2<F16>(p15, s2, b2);
    p26 = fma2<F16>(p26, s2, b2);
    p37 = fma2<F16>(p37, s2, b2);
    return make_uint4(pair_lo(p04, p15), pair_lo(p26, p37), pair_hi(p04, p15), pair_hi(p26, p37));
}

// Four 8-bit codes of one word -> (v0,v1), (v2,v3) as s*q+b.
template <bool F16>
QMM_DEVINL uint2 deq4_8bit(uint32_t w, uint32_t s2, uint32_t b2) {
    using H = Half<F16>;
    constexpr uint32_t MASK = 0x000F000Fu;
    const uint32_t one2 = H::kOne2;
    const uint32_t neg_off2 = F16 ? 0xE400E400u : 0xC300C300u;
    const uint32_t sixteen2 = F16 ? 0x4C004C00u : 0x41804180u;                         // (16, 16)
    const uint32_t lo02 = fma2<F16>(and_or(w, MASK, H::kMagic), one2, neg_off2);       // low nibbles of b0, b2
    const uint32_t hi02 = fma2<F16>(and_or(w >> 4, MASK, H::kMagic), one2, neg_off2);  // high nibbles
    const uint32_t lo13 = fma2<F16>(and_or(w >> 8, MASK, H::kMagic), one2, neg_off2);
    const uint32_t hi13 = fma2<F16>(and_or(w >> 12, MASK, H::kMagic), one2, neg_off2);
    uint32_t v02 = fma2<F16>(hi02, sixteen2, lo02);  // exact bytes (b0, b2)
    uint32_t v13 = fma2<F16>(hi13, sixteen2, lo13);
    v02 = fma2<F16>(v02, s2, b2);
    v13 = fma2<F16>(v13, s2, b2);
    return make_uint2(pair_lo(v02, v13), pair_hi(v02, v13));
}

// ---------------------------------------------------------------------------
// Variant with the dequantised weights in tensor memory (the A operand of
// tcgen05.mma read from TMEM, B = x from shared memory).
//
// Shared memory then holds only the TMA ring (x tile + packed codes), so the
// ring is deeper, and the bf16 weights never cross shared memory: each of
// the four dequantiser warps owns one 32-lane quarter of TMEM, one weight row
// per thread, and writes the row's 64 dequantised values of a k-block as 32
// consecutive columns (tcgen05.st 32x32b.x32; column c holds k = 2c, 2c+1).
// TMEM columns [0, BT) hold the fp32 accumulator, [BT, BT + 32*STAGES) the
// A stages.
// ---------------------------------------------------------------------------
template <int BITS, bool F16, int BT, int STAGES>
struct PfTmSmem {
    static constexpr int X_BYTES = BT * 128;
    static constexpr int P_BYTES = PF_BW * PF_BK * BITS / 8;
    static constexpr int X_OFF = 0;
    static constexpr int P_OFF = X_OFF + STAGES * X_BYTES;
    static constexpr int BAR_OFF = P_OFF + STAGES * P_BYTES;
    static constexpr int TOTAL = BAR_OFF + (4 * STAGES + 1) * 8 + 16 + 1024;
    static constexpr int A_COL = BT;  // first TMEM column of the A stages
    static constexpr int DQW = 8;     // dequantiser warps: two per TMEM lane quarter, one K half each
    static constexpr int THREADS = 64 + 32 * DQW;
    static constexpr int TMEM_COLS = 512;
    static_assert(BT + 32 * STAGES <= TMEM_COLS, "TMEM budget");
    static_assert(STAGES >= 3, "the dequantisers publish three k-blocks at a time");
};

template <int BITS, int GS, bool F16, int BT, int STAGES>
__global__ void __launch_bounds__(PfTmSmem<BITS, F16, BT, STAGES>::THREADS, 1)
    prefill_tm_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                      const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi, uint16_t* __restrict__ y,
                      int M, int N, int K) {
    using L = PfTmSmem<BITS, F16, BT, STAGES>;
    using H = Half<F16>;
    constexpr int WPR = PF_BK * BITS / 32;      // packed words per row per k-block (8 or 16)
    constexpr int VPG = GS < PF_BK ? GS : PF_BK;  // values of one group inside a k-block
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_base = sbase + L::BAR_OFF;
    auto full_x = [&](int s) { return bar_base + 8 * s; };
    auto full_p = [&](int s) { return bar_base + 8 * (STAGES + s); };
    auto a_ready = [&](int s) { return bar_base + 8 * (2 * STAGES + s); };
    auto empty = [&](int s) { return bar_base + 8 * (3 * STAGES + s); };
    const uint32_t acc_full = bar_base + 8 * (4 * STAGES);
    uint32_t* tmem_slot = (uint32_t*)(smem + L::BAR_OFF + (4 * STAGES + 1) * 8);
    volatile int* abort = (volatile int*)(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * PF_BW;
    const int m0 = blockIdx.y * BT;
    const int KB = (K + PF_BK - 1) / PF_BK;
    const int G = K / GS;
    const int kb_lo = 0, NKB = KB;  // this CTA's k-blocks

    if (threadIdx.x == 0) {
        *abort = 0;
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_x(s), 1);
            mbar_init(full_p(s), 1);
            mbar_init(a_ready(s), L::DQW);
            mbar_init(empty(s), 1);
        }
        mbar_init(acc_full, 1);
        mbar_fence_init();
        tma_prefetch_desc(&tmap_x);
        tma_prefetch_desc(&tmap_w);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(L::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        for (int i = 0; i < NKB; ++i) {  // warp-uniform loop, one elected lane issues
            const int kb = kb_lo + i, s = i % STAGES;
            const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
            mbar_wait(empty(s), ph ^ 1u, abort);
            if (elect_one()) {
                mbar_expect_tx(full_x(s), L::X_BYTES);
                tma_load_2d(sbase + L::X_OFF + s * L::X_BYTES, &tmap_x, full_x(s), kb * PF_BK, m0);
                mbar_expect_tx(full_p(s), L::P_BYTES);
                tma_load_2d(sbase + L::P_OFF + s * L::P_BYTES, &tmap_w, full_p(s), kb * WPR, n0);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: A from TMEM, B from shared memory ----------------
        // A warp-uniform loop with one elected lane issuing: issue from a
        // lane-0 branch rebuilds the operands in non-uniform registers and
        // cost ~100-200 cycles per MMA, which at four MMAs per k-block set the
        // k-block rate of the whole kernel.
        constexpr uint32_t idesc = PfIdesc<F16, BT>::value;
        const uint64_t bdesc0 = umma_desc_sw128(sbase + L::X_OFF);
        for (int i = 0; i < NKB; ++i) {
            const int s = i % STAGES;
            const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
            mbar_wait(full_x(s), ph, abort);
            mbar_wait(a_ready(s), ph, abort);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a_col = tmem + (uint32_t)(L::A_COL + 32 * s);
            // the B descriptor's address field counts 16-byte units
            const uint64_t bdesc = bdesc0 + (uint64_t)((s * L::X_BYTES) >> 4);
            if (elect_one()) {
#pragma unroll
                for (int kk = 0; kk < PF_BK / 16; ++kk)
                    umma_f16_ts(tmem, a_col + 8 * kk, bdesc + (uint64_t)((kk * 32) >> 4), idesc, (i | kk) != 0);
                umma_commit(empty(s));
            }
            __syncwarp();
        }
        if (elect_one()) umma_commit(acc_full);
        __syncwarp();
    } else {
        // ---------------- dequantisers (one weight row x one K half per thread), then epilogue ----------------
        constexpr int HW = WPR / 2;     // packed words of one K half
        constexpr int HV = PF_BK / 2;   // values of one K half (32)
        static_assert(HV <= VPG, "a K half lies inside one quantisation group (group size >= 32)");
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int half = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        int n = n0 + row;
        n = n < N ? n : N - 1;  // rows past N dequantise a valid row; their outputs are dropped
        const uint16_t* srow = sc + (long long)n * G;
        const uint16_t* brow = bi + (long long)n * G;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);

        // Scales and biases of three k-blocks in flight (rotated registers,
        // loop unrolled by three, each set refilled right after its use).
        auto fetch_sb = [&](int i, uint16_t& sv, uint16_t& bv) {
            const int k = (kb_lo + i) * PF_BK + half * HV;
            const int g = (i < NKB && k < K) ? k / GS : 0;
            sv = ldg_u16(srow + g);
            bv = ldg_u16(brow + g);
        };
        auto deq_block = [&](int i, uint16_t sv, uint16_t bv) {
            const int s = i % STAGES;
            const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
            const bool kval = (kb_lo + i) * PF_BK + half * HV < K;
            const uint32_t s2 = (uint32_t)sv | ((uint32_t)sv << 16);
            const uint32_t b2 = (uint32_t)bv | ((uint32_t)bv << 16);
            mbar_wait(full_p(s), ph, abort);
            mbar_wait(empty(s), ph ^ 1u, abort);  // the MMAs that read this A stage are done
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t* P =
                reinterpret_cast<const uint32_t*>(smem + L::P_OFF + s * L::P_BYTES) + row * WPR + half * HW;
            uint32_t wv[HW];
#pragma unroll
            for (int j = 0; j < HW; j += 4) {
                const uint4 pk = *reinterpret_cast<const uint4*>(P + j);
                wv[j] = pk.x;
                wv[j + 1] = pk.y;
                wv[j + 2] = pk.z;
                wv[j + 3] = pk.w;
            }
            uint32_t a[16];
#pragma unroll
            for (int j = 0; j < HW; ++j) {
                if constexpr (BITS == 4) {
                    uint4 v = deq8_4bit<F16>(wv[j], s2, b2);
                    if (!kval) v = make_uint4(0, 0, 0, 0);
                    a[4 * j] = v.x;
                    a[4 * j + 1] = v.y;
                    a[4 * j + 2] = v.z;
                    a[4 * j + 3] = v.w;
                } else {
                    uint2 v = deq4_8bit<F16>(wv[j], s2, b2);
                    if (!kval) v = make_uint2(0, 0);
                    a[2 * j] = v.x;
                    a[2 * j + 1] = v.y;
                }
            }
            tmem_st16(t_lane + (uint32_t)(L::A_COL + 32 * s + 16 * half), a);
        };
        // The stores of k-blocks i0 .. i0 + n - 1 are complete: hand those A
        // stages to the MMA (one store wait per three k-blocks).
        auto publish = [&](int i0, int n) {
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0)
                for (int j = 0; j < n; ++j) mbar_arrive(a_ready((i0 + j) % STAGES));
        };
        constexpr int STEP = 3;  // batches of three k-blocks
        uint16_t svA, bvA, svB, bvB, svC, bvC;
        const int i_first = 0;
        fetch_sb(i_first, svA, bvA);
        fetch_sb(i_first + 1, svB, bvB);
        fetch_sb(i_first + 2, svC, bvC);
        for (int i = i_first; i < NKB; i += STEP) {
            deq_block(i, svA, bvA);
            fetch_sb(i + STEP, svA, bvA);
            if (i + 1 < NKB) {
                deq_block(i + 1, svB, bvB);
                fetch_sb(i + STEP + 1, svB, bvB);
            }
            if (i + 2 < NKB) {
                deq_block(i + 2, svC, bvC);
                fetch_sb(i + STEP + 2, svC, bvC);
            }
            publish(i, NKB - i < 3 ? NKB - i : 3);
        }
        // ---------------- epilogue: TMEM -> y (each warp: its lane quarter, one half of the tokens) ----------------
        mbar_wait(acc_full, 0, abort);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int nout = n0 + row;
#pragma unroll 1
        for (int c0 = half * (BT / 2); c0 < (half + 1) * (BT / 2); c0 += 32) {
            uint32_t v[32];
            tmem_ld32(t_lane + (uint32_t)c0, v);
            tmem_wait_ld();
            if (nout < N) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int m = m0 + c0 + j;
                    if (m < M) y[(long long)m * N + nout] = H::from_f32(__uint_as_float(v[j]));
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS)
                     : "memory");
    }
}

}  // namespace qmm

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace qmm_host {

int prefill_supported(int bits, int gs) { return (bits == 4 || bits == 8) && (gs == 32 || gs == 64 || gs == 128); }

template <int BITS, int GS, bool F16, int BT, int STAGES>
static int launch_pf_tm(const CUtensorMap& mx, const CUtensorMap& mw, const uint16_t* sc, const uint16_t* bi,
                        uint16_t* y, long long M, long long N, long long K, cudaStream_t st) {
    using L = qmm::PfTmSmem<BITS, F16, BT, STAGES>;
    auto kern = qmm::prefill_tm_kernel<BITS, GS, F16, BT, STAGES>;
    {
        const int rc0 = ensure_smem_limit((const void*)kern, L::TOTAL, "prefill smem attribute");
        if (rc0) return rc0;
    }
    dim3 grid((unsigned)((N + qmm::PF_BW - 1) / qmm::PF_BW), (unsigned)((M + BT - 1) / BT));
    kern<<<grid, L::THREADS, L::TOTAL, st>>>(mx, mw, sc, bi, y, (int)M, (int)N, (int)K);
    return cuda_status(cudaGetLastError(), "prefill launch");
}

template <int BITS, int GS, bool F16>
static int launch_pf_bt(const CUtensorMap& mx, const CUtensorMap& mw, const uint16_t* sc, const uint16_t* bi,
                        uint16_t* y, long long M, long long N, long long K, int bt, cudaStream_t st) {
    // ring: x tile (BT x 64 x 2 B) + packed codes per stage within 227 KB; A stages in TMEM
    if (bt == 256) return launch_pf_tm<BITS, GS, F16, 256, BITS == 4 ? 6 : 5>(mx, mw, sc, bi, y, M, N, K, st);
    return launch_pf_tm<BITS, GS, F16, 128, BITS == 4 ? 8 : 8>(mx, mw, sc, bi, y, M, N, K, st);
}

int launch_prefill(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                   long long M, long long N, long long K, int gs, int bits, bool f16, cudaStream_t st, int force_bt) {
    int rc = QMM_OK;
    if (M > 65535LL * 128 || N > (1LL << 31) || K > (1LL << 31)) {
        set_error("prefill: shape M=%lld N=%lld K=%lld beyond limits", M, N, K);
        return QMM_EUNSUPPORTED;
    }
    const int bt = force_bt ? force_bt : (M <= 128 ? 128 : 256);
    CUtensorMap mx, mw;
    rc = tensor_map_2d(&mx, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, x, (uint64_t)K,
                       (uint64_t)M, (uint64_t)K * 2, 64, (uint32_t)bt, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t wrow = (uint64_t)K * bits / 32;
    rc = tensor_map_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, wrow, (uint64_t)N, wrow * 4, 64 * bits / 32,
                       qmm::PF_BW, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
#define QMM_PF_CASE(B, S)                                                                                      \
    if (bits == B && gs == S)                                                                                   \
        return f16 ? launch_pf_bt<B, S, true>(mx, mw, sc, bi, y, M, N, K, bt, st)                              \
                   : launch_pf_bt<B, S, false>(mx, mw, sc, bi, y, M, N, K, bt, st);
    QMM_PF_CASE(4, 32)
    QMM_PF_CASE(4, 64)
    QMM_PF_CASE(4, 128)
    QMM_PF_CASE(8, 32)
    QMM_PF_CASE(8, 64)
    QMM_PF_CASE(8, 128)
#undef QMM_PF_CASE
    set_error("prefill: bits=%d group_size=%d unsupported", bits, gs);
    return QMM_EUNSUPPORTED;
}

int qmv_device_error(int reset);
int qmv_sk_device_error(int reset);
int qmv_i8_device_error(int reset);

int device_error(int reset) {
    const int q0 = qmv_device_error(reset), q1 = qmv_sk_device_error(reset), q2 = qmv_i8_device_error(reset),
              q3 = moe_decode_device_error(reset);
    const int q = (q0 < 0 || q1 < 0 || q2 < 0 || q3 < 0) ? -1 : (q0 | q1 | q2 | q3);
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, qmm::g_dev_error, sizeof(int));
    if (e != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(qmm::g_dev_error, &z, sizeof(int));
    }
    return (q < 0 || v < 0) ? -1 : (v | q);
}

}  // namespace qmm_host
