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
#include "tc.cuh"
#include "tma.cuh"
#include "qmv_chunk.cuh"

namespace qmm {

template <int BITS, int GS, bool F16, int MT, int RW, bool GATHER, int STG_>
__global__ void __launch_bounds__(512, 1) qmv_kernel(const __grid_constant__ CUtensorMap wmap, QmvArgs args) {
    using G_ = QGeom<BITS, GS>;
    using R_ = QRing<BITS, GS, RW, STG_>;
    using H = Half<F16>;
    constexpr int WPT = G_::WPT, XR = G_::XR, STEPS = G_::STEPS, VPT = G_::VPT;
    constexpr int CH = G_::CH, CPG = G_::CPG, CPS = R_::CPS, STG = R_::STG;
    constexpr int CBU = R_::CHUNK_BYTES / 16;  // 16-byte units per chunk row (1, 2 or 4)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // stays shared-space

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int nwarps = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int N = args.N, K = args.K;
    const int G = K / GS;  // scale/bias groups per row
    const int C = K / CH;  // chunks per row

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + nwarps * R_::WARP_BYTES);
    volatile int* abort = reinterpret_cast<volatile int*>(bars + nwarps * STG);
    const uint32_t bar0 = smem_u32(bars + warp * STG);
    const uint32_t ring0 = smem_u32(smem + warp * R_::WARP_BYTES);

    pdl_launch_dependents();
    if (threadIdx.x == 0) *abort = 0;
    if (lane == 0) {
        for (int s = 0; s < STG; ++s) mbar_init(bar0 + 8 * s, 1);
        mbar_fence_init();
    }
    __syncthreads();

    // ---- rows of activations handled by this CTA ------------------------
    int m_count = args.M;
    int r0 = 0;
    int wrow0 = blockIdx.x * R_::ROWS;  // first weight row in the tensor map
    const uint16_t* sc = args.sc;
    const uint16_t* bi = args.bi;
    if constexpr (GATHER) {
        pdl_wait();  // the segment tables come from the previous kernel
        const Segments& sg = args.seg;
        const int item = blockIdx.y;
        const int total = ld_dep(sg.tile_prefix + sg.E);
        if (item >= total) return;
        // expert e with tile_prefix[e] <= item < tile_prefix[e+1]
        int lo = 0, hi = sg.E;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (ld_dep(sg.tile_prefix + mid) <= item) lo = mid; else hi = mid;
        }
        const int e = lo;
        const int chunk = item - ld_dep(sg.tile_prefix + e);
        r0 = ld_dep(sg.row_start + e) + 16 * chunk;
        m_count = min(16, ld_dep(sg.row_start + e + 1) - r0);
        wrow0 += e * N;
        sc += (long long)e * sg.s_stride;
        bi += (long long)e * sg.s_stride;
    }

    // ---- this warp's K range: whole TMA stages of CPS chunks ------------
    // Dense launches of gridDim.y = KC > 1 run as clusters of KC CTAs along y
    // that split K between their KC * nwarps warps (cluster rank = blockIdx.y).
    const int kc = GATHER ? 1 : (int)gridDim.y;
    const int kwarp = (GATHER ? 0 : (int)blockIdx.y) * nwarps + warp, nkw = kc * nwarps;
    const int SU = (C + CPS - 1) / CPS;
    const int ubase = SU / nkw, urem = SU % nkw;
    const int u0 = kwarp * ubase + min(kwarp, urem);
    const int nst = ubase + (kwarp < urem ? 1 : 0);
    const int g0 = u0 * CPS;
    const int ng = max(0, min(nst * CPS, C - g0));

    // one elected lane issues the copies from warp-uniform values (issue from
    // a lane-0 branch works on non-uniform registers and costs more per copy)
    auto issue = [&](int s, int st) {
        if (elect_one()) {
            mbar_expect_tx(bar0 + 8 * s, R_::STAGE_BYTES);
            tma_load_2d(ring0 + s * R_::STAGE_BYTES, &wmap, bar0 + 8 * s, (g0 + st * CPS) * G_::WPG, wrow0);
        }
        __syncwarp();
    };
    if (lane == 0) tma_prefetch_desc(&wmap);
    for (int s = 0; s < STG && s < nst; ++s) issue(s, s);
    if constexpr (!GATHER) pdl_wait();  // x comes from the previous kernel

    const int n_block = blockIdx.x * R_::ROWS;
    // per-stage bases of the scale/bias rows (advanced by CPS/CPG groups per stage)
    const uint16_t* sp[RW][2];
    const uint16_t* bp[RW][2];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            int n = n_block + 16 * r + g + 8 * h;
            n = n < N ? n : N - 1;  // rows past N read a valid row; their results are dropped
            sp[r][h] = sc + (long long)n * G + g0 / CPG;
            bp[r][h] = bi + (long long)n * G + g0 / CPG;
        }
    // per-stage base of the activation rows (advanced by CPS*CH values per stage)
    const uint16_t* xp[MT];
    bool xv[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = 8 * mt + g;
        xv[mt] = m < m_count;
        long long src = xv[mt] ? (long long)(r0 + m) : (long long)r0;
        if constexpr (GATHER) {
            if (args.seg.row_src != nullptr && xv[mt]) src = ld_dep(args.seg.row_src + r0 + m);
            if (src < 0 || src >= args.seg.x_rows) {  // out-of-range index: contribute zeros, read nothing
                xv[mt] = false;
                src = 0;
            }
        }
        xp[mt] = args.x + src * K + (long long)g0 * CH + t * VPT;
    }

    // thread-constant part of the swizzled shared-memory offset of a chunk
    const uint32_t tb = (uint32_t)t * WPT * 4;  // byte offset of the thread's words inside a chunk row
    const uint32_t tconst = ((((tb >> 4) ^ (uint32_t)g) & (CBU - 1)) << 4) | (tb & 15);
    const uint32_t hkey = (uint32_t)g & 7u & ~(uint32_t)(CBU - 1);
    const uint32_t rowbase = (uint32_t)g * 128;

    float res[RW][MT][4];
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) res[r][mt][c] = 0.0f;

    // activations, scales and biases of the next chunk (one chunk ahead)
    uint32_t xn[MT][XR];
    uint16_t sn[RW][2], bn[RW][2];
    auto fetch = [&](int xoff, int goff) {  // offsets from the current stage bases
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) load_x<XR>(xn[mt], xp[mt] + xoff, xv[mt]);
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                sn[r][h] = __ldg(sp[r][h] + goff);
                bn[r][h] = __ldg(bp[r][h] + goff);
            }
    };
    if (ng > 0) fetch(0, 0);

    for (int st = 0; st < nst; ++st) {
        const int s = st % STG;
        mbar_wait_bounded(bar0 + 8 * s, (uint32_t)(st / STG) & 1u, abort, &g_qmv_error);
        const uint32_t stage_addr = ring0 + s * R_::STAGE_BYTES + rowbase;
#pragma unroll
        for (int c = 0; c < CPS; ++c) {
            const int i = st * CPS + c;
            if (i < ng) {
                uint32_t xr[MT][XR];
                float s_[RW][2], b_[RW][2];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int k = 0; k < XR; ++k) xr[mt][k] = xn[mt][k];
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        s_[r][h] = H::to_f32(sn[r][h]);
                        b_[r][h] = H::to_f32(bn[r][h]);
                    }
                if (i + 1 < ng) fetch((c + 1) * CH, (c + 1) / CPG);

                // packed words of rows g and g+8 of every tile from the swizzled stage
                uint32_t wv[RW][2][WPT];
                const uint32_t cofs = (((((uint32_t)(c * CBU)) ^ hkey) & 7u) << 4) | tconst;
                lds_tile_rows<RW, WPT>(stage_addr + cofs, wv);

                chunk_math<BITS, F16, MT, RW, XR, WPT, STEPS>(res, xr, wv, s_, b_);
            }
        }
        // advance the per-stage bases
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) xp[mt] += CPS * CH;
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                sp[r][h] += CPS / CPG;
                bp[r][h] += CPS / CPG;
            }
        __syncwarp();  // every lane is done with stage s
        if (st + STG < nst) issue(s, st + STG);
    }

    // ---- fixed-order reduction of the K slices (reuses the ring memory) ----
    constexpr int NV = RW * MT * 4;
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);  // [nwarps][NV][32]
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) red[((warp * NV) + (r * MT + mt) * 4 + c) * 32 + lane] = res[r][mt][c];
    __syncthreads();
    // each CTA sums its own warps in warp order, in place (thread idx alone
    // reads and then writes the warp-0 slot of its element)
    for (int idx = threadIdx.x; idx < NV * 32; idx += blockDim.x) {
        const int ln = idx & 31, v = idx >> 5;
        float sum = 0.0f;
        for (int wk = 0; wk < nwarps; ++wk) sum += red[(wk * NV + v) * 32 + ln];
        red[v * 32 + ln] = sum;
    }
    // a cluster: every CTA's sums are written and visible before rank 0 reads
    // them (every thread of every CTA reaches this point: no early exit in the
    // dense path, and every wait above is bounded)
    if (kc > 1) {
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
    const uint32_t red_s = smem_u32(red);
    const bool sums = kc == 1 || blockIdx.y == 0;  // a cluster's rank 0 adds the ranks in order and stores
    for (int idx = threadIdx.x; sums && idx < NV * 32; idx += blockDim.x) {
        const int ln = idx & 31, v = idx >> 5;
        float sum = red[v * 32 + ln];
        for (int q = 1; q < kc; ++q) {
            uint32_t remote;
            float val;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(red_s + (uint32_t)((v * 32 + ln) * 4)), "r"(q));
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(val) : "r"(remote) : "memory");
            sum += val;
        }
        const int c = v & 3, mt = (v >> 2) % MT, r = (v >> 2) / MT;
        const int gg = ln >> 2, tt = ln & 3;
        const int n = n_block + 16 * r + gg + 8 * (c >> 1);
        const int m = 8 * mt + 2 * tt + (c & 1);
        if (n < N && m < m_count) {
            long long dst = r0 + m;
            if constexpr (GATHER) {
                if (args.seg.row_scale != nullptr) sum *= ld_dep(args.seg.row_scale + r0 + m);
                if (args.seg.row_dst != nullptr) dst = ld_dep(args.seg.row_dst + r0 + m);
                if (dst < 0 || dst >= args.seg.y_rows) continue;
            }
            args.y[dst * N + n] = H::from_f32(sum);
        }
    }
    // the other ranks' shared memory stays alive until rank 0 has read it
    if (kc > 1) {
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
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

// For N <= 1024 (at most 64 16-row tiles, so 84+ SMs would sit idle) each
// tile's K is split across a cluster of two CTAs of 10 warps, each CTA sums
// its warps in order and rank 0 adds rank 1's sums over DSMEM: 1024x5120 at
// M = 1 / 4 / 8 / 16 takes 4.19 / 4.33 / 4.44 / 4.96 us against 4.28 / 4.36 /
// 4.52 / 5.70 us on one CTA of 12 warps (at N = 2048 one CTA stays faster).
// Matrices this CTA-per-tile kernel serves faster than the stream-K kernel
// when the caller gives a workspace: 4-bit codes in groups of 64, K <= 5632
// (at most 88 K chunks, so the split over 8 or 12 warps stays short) and
// fewer than 24 MiB of codes (M <= 8 calls on 12 MiB and more take the
// integer-MMA kernel first).  Measured on B200 (CUDA graphs, PDL), M = 1..16,
// K = 5120: N = 1024 / 2048 / 4096 / 6144 / 8192 take 4.3 / 4.9 / 6.7 / 9.3 /
// 9.8 us against 6.5 / 7.3 / 9.0 / 10.6 / 12.7 us for the stream-K kernel,
// whose fix-up of split tiles costs more than a shared-memory reduction at
// these sizes; at K = 6144 they tie and at K = 8192 stream-K is faster.  The
// choice depends on the matrix only, so every M <= 16 call on one matrix
// takes the same kernel and tile shape (rows keep single-row bits).
bool qmv_cta_preferred(long long N, long long K, int gs, int bits, int* rw, int* kw, int* kc) {
    if (bits != 4 || gs != 64 || K > 5632 || N * K * bits / 8 >= (24LL << 20)) return false;
    *rw = N <= 2048 ? 1 : 2;
    *kw = N <= 1024 ? 10 : N <= 4096 ? 12 : 8;
    *kc = N <= 1024 ? 2 : 1;  // at most 64 row tiles: two CTAs (a cluster) per tile split K
    return true;
}

// M = 9..16 on matrices of 24 MiB of codes and more with K <= 5632 (groups
// of 64, 4- or 8-bit codes): this kernel with 32-row tiles and 4 K-warps.
// Measured on B200 (CUDA graphs, PDL), M = 9 / 16: 17408x5120 4-bit 24.1 /
// 24.4 us against 30.4 / 31.3 us for the stream-K kernel, the 8-bit
// 248320x5120 lm_head 411 / 397 us against 498 / 525 us; at K = 17408 and
// K = 6144 stream-K stays faster.  Rows of M = 9..16 calls share one schedule
// among themselves (the M <= 8 rule above is unchanged).
bool qmv_cta_preferred_wide(long long N, long long K, int gs, int bits, int* rw, int* kw) {
    if ((bits != 4 && bits != 8) || gs != 64 || K > 5632 || N * K * bits / 8 < (24LL << 20)) return false;
    *rw = 2;
    *kw = 4;
    return true;
}

template <int BITS, int GS, bool F16, int MT, int RW, bool GATHER, int STG_ = 0>
static int launch_qmv_t(const QmvArgs& a, int k_warps, int grid_y, long long w_rows, cudaStream_t st) {
    using R_ = qmm::QRing<BITS, GS, RW, STG_>;
    auto kern = qmm::qmv_kernel<BITS, GS, F16, MT, RW, GATHER, STG_>;
    const int threads = 32 * k_warps;
    const size_t ring = (size_t)k_warps * R_::WARP_BYTES;
    const size_t red = (size_t)k_warps * RW * MT * 4 * 32 * sizeof(float);
    const size_t smem = (ring > red ? ring : red) + (size_t)k_warps * R_::STG * 8 + 16 + 1024;
    int rc0 = ensure_smem_limit((const void*)kern, 227 * 1024, "qmv smem attribute");
    if (rc0) return rc0;
    CUtensorMap wmap;
    const uint64_t wrow = (uint64_t)a.K * BITS / 32;
    int rc = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, a.w, wrow, (uint64_t)w_rows, wrow * 4, 32,
                           (uint32_t)R_::ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.N + R_::ROWS - 1) / R_::ROWS), (unsigned)grid_y, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[2];
    int na = 0;
    if (pdl_enabled()) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (!GATHER && grid_y > 1) {  // the K split across a cluster of grid_y CTAs
        if (grid_y > 8) {
            set_error("qmv: a K split over %d CTAs exceeds the portable cluster size", grid_y);
            return QMM_EINVAL;
        }
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = 1;
        attrs[na].val.clusterDim.y = (unsigned)grid_y;
        attrs[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    if (smem > 227 * 1024) {
        set_error("qmv: %d K-split warps need %zu bytes of shared memory", k_warps, smem);
        return QMM_EINVAL;
    }
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wmap, a);
    if (e != cudaSuccess) cudaGetLastError();  // a failed launch must not leave a stale error behind
    return cuda_status(e, "qmv launch");
}

template <int BITS, int GS, bool F16, bool GATHER>
static int launch_qmv_mt(const QmvArgs& a, int mt, int rw, int k_warps, int grid_y, long long w_rows,
                         cudaStream_t st) {
    if (mt == 1) {
        return rw == 1 ? launch_qmv_t<BITS, GS, F16, 1, 1, GATHER>(a, k_warps, grid_y, w_rows, st)
                       : launch_qmv_t<BITS, GS, F16, 1, 2, GATHER>(a, k_warps, grid_y, w_rows, st);
    }
    return rw == 1 ? launch_qmv_t<BITS, GS, F16, 2, 1, GATHER>(a, k_warps, grid_y, w_rows, st)
                   : launch_qmv_t<BITS, GS, F16, 2, 2, GATHER>(a, k_warps, grid_y, w_rows, st);
}

// Tuning hook: explicit ring depth for the 4-bit g64 bf16 kernel.
int launch_qmv_stages(const QmvArgs& a, int mt, int rw, int k_warps, int stages, cudaStream_t st) {
    const long long w_rows = a.N;
#define QMM_STG(S)                                                                                             \
    if (stages == S) {                                                                                          \
        if (mt == 1) return rw == 1 ? launch_qmv_t<4, 64, false, 1, 1, false, S>(a, k_warps, 1, w_rows, st)     \
                                    : launch_qmv_t<4, 64, false, 1, 2, false, S>(a, k_warps, 1, w_rows, st);    \
        return rw == 1 ? launch_qmv_t<4, 64, false, 2, 1, false, S>(a, k_warps, 1, w_rows, st)                 \
                       : launch_qmv_t<4, 64, false, 2, 2, false, S>(a, k_warps, 1, w_rows, st);                \
    }
    QMM_STG(2)
    QMM_STG(3)
    QMM_STG(4)
    QMM_STG(6)
#undef QMM_STG
    set_error("stages=%d not instantiated", stages);
    return QMM_EINVAL;
}

template <bool GATHER>
int launch_qmv(const QmvArgs& a, int bits, int gs, bool f16, int mt, int rw, int k_warps, int grid_y,
               cudaStream_t st) {
    const long long w_rows = GATHER ? (long long)a.seg.E * a.N : (long long)a.N;
#define QMM_QMV_CASE(B, S)                                                                               \
    if (bits == B && gs == S)                                                                             \
        return f16 ? launch_qmv_mt<B, S, true, GATHER>(a, mt, rw, k_warps, grid_y, w_rows, st)           \
                   : launch_qmv_mt<B, S, false, GATHER>(a, mt, rw, k_warps, grid_y, w_rows, st);
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

int qmv_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, qmm::g_qmv_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(qmm::g_qmv_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace qmm_host
