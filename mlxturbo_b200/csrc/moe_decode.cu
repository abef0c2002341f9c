// moe_decode.cu -- the MoE block at decode widths in one launch:
//
//   y[t] = sum_k w[t,k] * down_e(silu(gate_e x_t) * up_e x_t),   e = ids[t,k]
//
// for T tokens and top_k routed experts each: the SparseMoeBlock of
// mlxturbo/_vendor/qwen4_exp.py:1763-1806 over the SwitchGLU banks, which the
// reference runs as gather_qmv per projection plus glue (sort, combine).
//
// Phase A (gate/up and SwiGLU).  A unit is one (token, expert) pair and one
// 16-row block of the interleaved gate/up bank (gate rows of channels
// 8b..8b+7, then the up rows of the same channels) over all of K = hidden.
// CTA c takes units c, c + G, ..., so a small launch spreads them over every
// SM; when a CTA has fewer units than warps, each unit's K range is cut into
// KS slices (items) that run on different warps and meet in shared memory
// (T = 1: 640 units, two slices each, on 1776 warps).  The lane holding
// column 0 of rows g and g+8 has the gate and up value of channel 8b+g;
// silu(gate)*up, rounded to the activation dtype, goes to the pair's row of h
// (a workspace array, L2-resident).
//
// Phase B (down and combine).  A unit is one token and 16 output rows.  The
// CTA's warps split the token's top_k pairs; each streams its pair's expert's
// 16 down rows over K = intermediate against the pair's h row and weights the
// result by the router weight.  The CTA adds the warps' sums in warp order,
// so y does not depend on timing, and stores 16 values of y.
//
// One grid barrier separates the phases: one CTA of 12 warps per SM, every CTA
// resident (the grid is the SM count and the host checks that one CTA fits).
// The weights of both phases stream through one TMA ring per warp as a single
// sequence of stages, so a warp's first down-projection stages (which do not
// depend on h) are issued as soon as its phase-A stages free ring slots:
// at T = 1 most of the down weights are in shared memory before the barrier.
//
// Pairs are not grouped by expert (no sort): at T = 1 the ten pairs name ten
// experts; at larger T an expert chosen by two tokens is read twice, the
// reference's own gather_qmv behaviour.  The host takes this kernel for small
// T only (the library's four-launch block reads each expert once).
//
// Waits are bounded: an mbarrier wait or the grid barrier that gives up sets
// the device error flag (qmm_device_error) and the kernel runs to its end.

#include "qmv_chunk.cuh"
#include "tc.cuh"
#include "tma.cuh"

namespace qmm {

__device__ int g_md_error;

constexpr int kMdWarps = 12;  // warps per CTA (one CTA per SM)
constexpr int kMdStages = 4;  // ring stages per warp
constexpr int kMdScBox = 256;  // bytes of one 8-group x 16-row box of scales (or biases)
constexpr int kMdMaxSlots = 64;  // phase-A (unit, slice) items of one CTA whose partials are kept

struct MdArgs {
    const uint16_t* x;        // [T, H] activations
    const int* ids;           // [T * top_k] expert of each pair (token-major)
    const float* wts;         // [T * top_k] router weight of each pair
    uint16_t* y;              // [T, H]
    uint16_t* h;              // [T * top_k, I] SwiGLU output per pair (workspace)
    unsigned long long* ctr;  // grid-barrier arrivals (workspace; a multiple of the grid between calls)
    int T, top_k, E, H, I;
    int UA, UB;  // phase-A units (pairs x I/8 blocks), phase-B CTA units (T x H/16)
    int KS;      // K slices per phase-A unit (divides H / stage K; > 1 when units are fewer than warps)
};

// Shared-memory layout (byte offsets from a 1024-aligned base).
struct MdLayout {
    uint32_t ring, scl, xs, hb, red, ids, wts, bars, abort, total;
};

template <int BITS, int GS>
__host__ __device__ inline MdLayout md_layout(int T, int H, int I, int P) {
    using R_ = QRing<BITS, GS, 1, kMdStages>;
    MdLayout L;
    uint32_t o = 0;
    L.ring = o;
    o += kMdWarps * kMdStages * R_::STAGE_BYTES;
    L.scl = o;
    o += kMdWarps * kMdStages * 2 * kMdScBox;
    L.xs = o;
    o += ((uint32_t)(T * H * 2) + 15u) & ~15u;
    L.hb = o;
    o += kMdWarps * 2 * I * 2;
    L.red = o;
    o += kMdMaxSlots * 16 * 4;  // phase-A slice partials, or phase-B warp sums (kMdWarps x 16)
    L.ids = o;
    o += ((uint32_t)(P * 4) + 15u) & ~15u;
    L.wts = o;
    o += ((uint32_t)(P * 4) + 15u) & ~15u;
    L.bars = o;
    o += kMdWarps * kMdStages * 8;
    L.abort = o;
    o += kMdWarps * 4;
    L.total = o + 1024;  // alignment slack of the dynamic shared memory base
    return L;
}

QMM_DEVINL unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

QMM_DEVINL uint4 ld_cg_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

template <int BITS, int GS, bool F16>
__global__ void __launch_bounds__(32 * kMdWarps, 1)
    moe_glu_decode_kernel(const __grid_constant__ CUtensorMap guw, const __grid_constant__ CUtensorMap gus,
                          const __grid_constant__ CUtensorMap gub, const __grid_constant__ CUtensorMap dnw,
                          const __grid_constant__ CUtensorMap dns, const __grid_constant__ CUtensorMap dnb,
                          MdArgs a) {
    using G_ = QGeom<BITS, GS>;
    using R_ = QRing<BITS, GS, 1, kMdStages>;
    using H_ = Half<F16>;
    constexpr int WPT = G_::WPT, XR = G_::XR, STEPS = G_::STEPS, VPT = G_::VPT, CH = G_::CH, CPG = G_::CPG;
    constexpr int CPS = R_::CPS, STG = kMdStages;
    constexpr int SK = CPS * CH;        // K values per stage
    constexpr int GPS = CPS / CPG;      // quantisation groups per stage (1, 2, 4 or 8)
    constexpr int CBU = R_::CHUNK_BYTES / 16;
    constexpr int WPS = SK * BITS / 32;  // packed words per row per stage (32)
    static_assert(GPS >= 1 && 8 % GPS == 0, "a stage's groups lie in one 8-group box");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int P = a.T * a.top_k;
    const MdLayout L = md_layout<BITS, GS>(a.T, a.H, a.I, P);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int G = gridDim.x;
    // Phase A: CTA c owns units c, c + G, ... (every SM gets work when units
    // are fewer than warps), each cut into KS slices of SA / KS stages; item
    // i = j * KS + q of the CTA (its j-th unit, slice q) goes to warp
    // i % kMdWarps.  With KS > 1 the slices' partial sums meet in shared
    // memory and the SwiGLU runs after the CTA's items: a unit's K range
    // split over KS warps shortens the one serial chain that bounds a small
    // launch (T = 1: 640 units, 1776 warps).
    const int nA = blockIdx.x < a.UA ? (a.UA - 1 - blockIdx.x) / G + 1 : 0;  // this CTA's units
    const int nItems = nA * a.KS;
    const int NBA = a.I / 8;   // 16-row blocks of the fused gate/up bank per expert
    const int NBB = a.H / 16;  // 16-row blocks of the down bank per expert
    const int SA = a.H / SK, SB = a.I / SK;
    const int SPS = SA / a.KS;  // stages per phase-A slice

    const uint32_t ring0 = smem_u32(smem + L.ring) + warp * STG * R_::STAGE_BYTES;
    uint8_t* sring = smem + L.scl + warp * STG * 2 * kMdScBox;
    const uint32_t bar0 = smem_u32(smem + L.bars) + warp * STG * 8;
    volatile int* abort = reinterpret_cast<volatile int*>(smem + L.abort) + warp;
    int* ids_s = reinterpret_cast<int*>(smem + L.ids);
    float* wts_s = reinterpret_cast<float*>(smem + L.wts);
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + L.xs);
    float* red = reinterpret_cast<float*>(smem + L.red);
    uint16_t* hb = reinterpret_cast<uint16_t*>(smem + L.hb) + warp * 2 * a.I;

    pdl_launch_dependents();
    if (lane == 0) {
        *abort = 0;
        for (int s = 0; s < STG; ++s) mbar_init(bar0 + 8 * s, 1);
        mbar_fence_init();
    }
    if (threadIdx.x == 0) {
        tma_prefetch_desc(&guw);
        tma_prefetch_desc(&gus);
        tma_prefetch_desc(&gub);
        tma_prefetch_desc(&dnw);
        tma_prefetch_desc(&dns);
        tma_prefetch_desc(&dnb);
    }
    pdl_wait();  // ids, router weights and x come from earlier work (a no-op under the plain launch)
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        ids_s[i] = ld_dep(a.ids + i);
        wts_s[i] = ld_dep(a.wts + i);
    }
    __syncthreads();

    // expert of pair p for addressing (an id outside [0, E) reads expert 0;
    // its contribution is dropped below)
    auto expert = [&](int p) {
        const int e = ids_s[p];
        return (e >= 0 && e < a.E) ? e : 0;
    };

    // The issue cursor walks this warp's stages in consumption order: its
    // phase-A items (warp, warp + kMdWarps, ...) x SPS stages, then for each of the CTA's
    // phase-B units (blockIdx.x, + G, ...) its pairs (k = warp, + 8, ...) x SB
    // stages.  Warp-uniform state; one elected lane issues the copies.
    int c_ph, c_u, c_k, c_ks;  // phase (0 A, 1 B, 2 done), unit, pair slot, stage
    auto b_norm = [&]() {
        while (c_ph == 1) {
            if (c_u >= a.UB) {
                c_ph = 2;
                break;
            }
            if (c_k < a.top_k) break;
            c_u += G;
            c_k = warp;
        }
    };
    auto enter_b = [&]() {
        c_ph = 1;
        c_u = blockIdx.x;
        c_k = warp;
        c_ks = 0;
        b_norm();
    };
    c_ks = 0;
    c_k = warp;
    if (warp < nItems) {
        c_ph = 0;
        c_u = warp;  // phase A: the CTA item index
    } else {
        enter_b();
    }
    auto issue = [&](int s) {
        int row;
        const CUtensorMap *wm, *sm, *bm;
        int ks = c_ks;
        if (c_ph == 0) {
            const int u = blockIdx.x + (c_u / a.KS) * G;
            const int p = u / NBA, b = u - p * NBA;
            row = expert(p) * 2 * a.I + 16 * b;
            ks += (c_u % a.KS) * SPS;
            wm = &guw;
            sm = &gus;
            bm = &gub;
        } else {
            const int tok = c_u / NBB, c = c_u - tok * NBB;
            row = expert(tok * a.top_k + c_k) * a.H + 16 * c;
            wm = &dnw;
            sm = &dns;
            bm = &dnb;
        }
        if (++c_ks == (c_ph == 0 ? SPS : SB)) {
            c_ks = 0;
            if (c_ph == 0) {
                c_u += kMdWarps;
                if (c_u >= nItems) enter_b();
            } else {
                c_k += kMdWarps;
                b_norm();
            }
        }
        if (elect_one()) {
            mbar_expect_tx(bar0 + 8 * s, R_::STAGE_BYTES + 2 * kMdScBox);
            tma_load_2d(ring0 + s * R_::STAGE_BYTES, wm, bar0 + 8 * s, ks * WPS, row);
            // the stage's groups inside the 8-group box at the boundary below
            const int gx = (ks * GPS) & ~7;
            const uint32_t sdst = smem_u32(sring) + s * 2 * kMdScBox;
            tma_load_2d(sdst, sm, bar0 + 8 * s, gx, row);
            tma_load_2d(sdst + kMdScBox, bm, bar0 + 8 * s, gx, row);
        }
        __syncwarp();
    };
    for (int s = 0; s < STG && c_ph != 2; ++s) issue(s);

    // x into shared memory while the first stages are in flight
    {
        const int nx = a.T * a.H / 8;
        const uint4* src = reinterpret_cast<const uint4*>(a.x);
        uint4* dst = reinterpret_cast<uint4*>(xs);
        for (int i = threadIdx.x; i < nx; i += blockDim.x) dst[i] = ld_v4(src + i);
    }
    __syncthreads();

    const uint32_t tb = (uint32_t)t4 * WPT * 4;
    const uint32_t tconst = ((((tb >> 4) ^ (uint32_t)g) & (CBU - 1)) << 4) | (tb & 15);
    const uint32_t hkey = (uint32_t)g & 7u & ~(uint32_t)(CBU - 1);
    const uint32_t rowbase = (uint32_t)g * 128;
    float res[1][1][4];
    int st = 0;  // stages consumed (ring position)

    // Stage `ks` of the current unit against the activation row at shared
    // address xa (the stage's K values start at xa + ks * SK * 2).  Every
    // lane reads the same row: MMA columns 1..7 repeat column 0 and are
    // dropped.
    auto consume = [&](uint32_t xa, int ks) {
        const int s = st % STG;
        mbar_wait_bounded(bar0 + 8 * s, (uint32_t)(st / STG) & 1u, abort, &g_md_error);
        const uint32_t stage_addr = ring0 + s * R_::STAGE_BYTES + rowbase;
        const uint16_t* sp = reinterpret_cast<const uint16_t*>(sring + s * 2 * kMdScBox) + g * 8;
        const uint32_t xk = xa + (uint32_t)(ks * SK * 2);
        unroll_chunks<CPS>([&](auto cc) {
            constexpr int c = decltype(cc)::value;
            uint32_t xr[1][XR];
            const uint32_t xaddr = xk + (uint32_t)((c * CH + t4 * VPT) * 2);
#pragma unroll
            for (int i = 0; i < XR; i += 4)
                asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                             : "=r"(xr[0][i]), "=r"(xr[0][i + 1]), "=r"(xr[0][i + 2]), "=r"(xr[0][i + 3])
                             : "r"(xaddr + 4 * i));
            float s_[1][2], b_[1][2];
            const int gi = ((ks * GPS) & 7) + c / CPG;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                s_[0][hh] = H_::to_f32(sp[8 * hh * 8 + gi]);
                b_[0][hh] = H_::to_f32(sp[kMdScBox / 2 + 8 * hh * 8 + gi]);
            }
            uint32_t wv[1][2][WPT];
            const uint32_t cofs = (((((uint32_t)(c * CBU)) ^ hkey) & 7u) << 4) | tconst;
            lds_tile_rows<1, WPT>(stage_addr + cofs, wv);
            chunk_math<BITS, F16, 1, 1, XR, WPT, STEPS>(res, xr, wv, s_, b_);
        });
        __syncwarp();  // every lane is done with slot s before it is refilled
        if (c_ph != 2) issue(s);
        ++st;
    };

    // ---- phase A: h[p][8b + g] = silu(gate) * up ------------------------------
    for (int i = warp; i < nItems; i += kMdWarps) {
        const int u = blockIdx.x + (i / a.KS) * G;
        const int p = u / NBA, b = u - p * NBA;
        const int tok = p / a.top_k;
        res[0][0][0] = res[0][0][1] = res[0][0][2] = res[0][0][3] = 0.0f;
        const uint32_t xrow = smem_u32(xs) + (uint32_t)(tok * a.H * 2);
        const int k0 = (i % a.KS) * SPS;
        for (int ks = k0; ks < k0 + SPS; ++ks) consume(xrow, ks);
        if (t4 == 0) {
            if (a.KS == 1) {
                const int e = ids_s[p];
                float v = 0.0f;
                if (e >= 0 && e < a.E) {
                    const float gt = res[0][0][0], up = res[0][0][2];
                    v = gt / (1.0f + expf(-gt)) * up;
                }
                a.h[(size_t)p * a.I + 8 * b + g] = H_::from_f32(v);
            } else {
                red[i * 16 + g] = res[0][0][0];
                red[i * 16 + 8 + g] = res[0][0][2];
            }
        }
    }
    if (a.KS > 1) {  // the slices' sums in slice order, then the SwiGLU
        __syncthreads();
        for (int j = warp; j < nA; j += kMdWarps) {
            if (lane < 8) {
                float gt = 0.0f, up = 0.0f;
                for (int q = 0; q < a.KS; ++q) {
                    gt += red[(j * a.KS + q) * 16 + lane];
                    up += red[(j * a.KS + q) * 16 + 8 + lane];
                }
                const int u = blockIdx.x + j * G;
                const int p = u / NBA, b = u - p * NBA;
                const int e = ids_s[p];
                float v = 0.0f;
                if (e >= 0 && e < a.E) v = gt / (1.0f + expf(-gt)) * up;
                a.h[(size_t)p * a.I + 8 * b + lane] = H_::from_f32(v);
            }
        }
    }

    // ---- grid barrier: every pair's h row is written ---------------------------
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned long long old = atomicAdd(a.ctr, 1ull);
        const unsigned long long target = old - old % (unsigned long long)G + (unsigned long long)G;
        bool ok = false;
        for (uint32_t i = 0; i < (1u << 22); ++i) {
            if (ld_acquire_u64(a.ctr) >= target) {
                ok = true;
                break;
            }
            __nanosleep(64);
        }
        if (!ok) atomicExch(&g_md_error, 2);
        __threadfence();
    }
    __syncthreads();

    // ---- phase B: y[tok][16c + r] = sum_k w * (down_e rows . h) ----------------
    const int hv = a.I / 256;  // 16-byte vectors of one h row per lane (I * 2 bytes / 32 lanes)
    int hbuf = 0;
    uint4 hn[8];
    for (int u = blockIdx.x; u < a.UB; u += G) {
        const int tok = u / NBB, c = u - tok * NBB;
        auto load_h = [&](int k) {
            const uint4* src = reinterpret_cast<const uint4*>(a.h + (size_t)(tok * a.top_k + k) * a.I) + lane;
#pragma unroll
            for (int v = 0; v < 8; ++v)
                if (v < hv) hn[v] = ld_cg_v4(src + 32 * v);
        };
        auto store_h = [&](int buf) {
            uint4* dst = reinterpret_cast<uint4*>(hb + buf * a.I) + lane;
#pragma unroll
            for (int v = 0; v < 8; ++v)
                if (v < hv) dst[32 * v] = hn[v];
        };
        float acc0 = 0.0f, acc1 = 0.0f;
        int k = warp;
        if (k < a.top_k) {
            load_h(k);
            store_h(hbuf);
        }
        __syncwarp();
        for (; k < a.top_k; k += kMdWarps) {
            const int kn = k + kMdWarps;
            if (kn < a.top_k) load_h(kn);  // the next pair's h row, in flight while this pair's stages run
            const int p = tok * a.top_k + k;
            res[0][0][0] = res[0][0][1] = res[0][0][2] = res[0][0][3] = 0.0f;
            const uint32_t xrow = smem_u32(hb + hbuf * a.I);
            for (int ks = 0; ks < SB; ++ks) consume(xrow, ks);
            const int e = ids_s[p];
            const float wk = (e >= 0 && e < a.E) ? wts_s[p] : 0.0f;
            acc0 = fmaf(wk, res[0][0][0], acc0);
            acc1 = fmaf(wk, res[0][0][2], acc1);
            if (kn < a.top_k) {
                store_h(hbuf ^ 1);
                hbuf ^= 1;
            }
            __syncwarp();
        }
        if (t4 == 0) {
            red[warp * 16 + g] = acc0;
            red[warp * 16 + 8 + g] = acc1;
        }
        __syncthreads();
        if (warp == 0 && lane < 16) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kMdWarps; ++w) v += red[w * 16 + lane];
            a.y[(size_t)tok * a.H + 16 * c + lane] = H_::from_f32(v);
        }
        __syncthreads();
    }
}

}  // namespace qmm

// ---------------------------------------------------------------------------
// host launch
// ---------------------------------------------------------------------------
namespace qmm_host {

int moe_decode_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, qmm::g_md_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(qmm::g_md_error, &z, sizeof(int));
    }
    return v;
}

size_t moe_decode_workspace(long long T, long long top_k, long long I) {
    return 256 + (size_t)T * (size_t)top_k * (size_t)I * 2;
}

// The shapes the kernel takes (else QMM_EUNSUPPORTED: the caller runs the
// block as separate launches).
int moe_decode_supported(long long T, long long top_k, long long E, long long H, long long I, int gs, int bits) {
    // K values per ring stage (1024 / bits); the h rows are staged as 16-byte
    // vectors of 32 lanes, so inter is a multiple of 256 for either width
    const long long SK = 1024 / bits;
    if (H % SK || I % 256 || (H / gs) % 8 || (I / gs) % 8) {
        set_error("moe_glu_decode: hidden=%lld must be a multiple of %lld and intermediate=%lld of 256, with a "
                  "multiple of 8 quantisation groups per row",
                  H, SK, I);
        return QMM_EUNSUPPORTED;
    }
    if (I > 2048 || T * H * 2 > 32768 || T * top_k > 1024 || E * 2 * I >= (1LL << 31) || E * H >= (1LL << 31)) {
        set_error("moe_glu_decode: T=%lld top_k=%lld hidden=%lld intermediate=%lld outside the one-launch block "
                  "(intermediate <= 2048, T * hidden <= 16384, T * top_k <= 1024)",
                  T, top_k, H, I);
        return QMM_EUNSUPPORTED;
    }
    return QMM_OK;
}

template <int BITS, int GS, bool F16>
static int launch_md_t(const MoeDecodeCall& c) {
    auto kern = qmm::moe_glu_decode_kernel<BITS, GS, F16>;
    const int P = c.T * c.top_k;
    const qmm::MdLayout L = qmm::md_layout<BITS, GS>(c.T, c.H, c.I, P);
    int dev = 0, optin = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        cudaGetLastError();
        set_error("moe_glu_decode: device query failed");
        return QMM_ECUDA;
    }
    if ((int)L.total > optin) {
        set_error("moe_glu_decode: %u bytes of shared memory per CTA exceed the device's %d", L.total, optin);
        return QMM_EUNSUPPORTED;
    }
    int rc = ensure_smem_limit((const void*)kern, (int)L.total, "moe_glu_decode smem attribute");
    if (rc) return rc;
    // the grid barrier needs every CTA resident: one per SM, and one must fit
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 32 * qmm::kMdWarps, L.total) != cudaSuccess ||
        occ < 1) {
        cudaGetLastError();
        set_error("moe_glu_decode: no resident CTA of %d warps with %u bytes of shared memory", qmm::kMdWarps,
                  L.total);
        return QMM_EUNSUPPORTED;
    }
    const CUtensorMapDataType dt = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap guw, gus, gub, dnw, dns, dnb;
    const uint64_t gu_rows = (uint64_t)c.E * 2 * c.I, dn_rows = (uint64_t)c.E * c.H;
    const uint64_t gu_words = (uint64_t)c.H * BITS / 32, dn_words = (uint64_t)c.I * BITS / 32;
    const uint64_t gu_groups = (uint64_t)c.H / GS, dn_groups = (uint64_t)c.I / GS;
    if ((rc = tensor_map_2d(&guw, CU_TENSOR_MAP_DATA_TYPE_UINT32, c.guw, gu_words, gu_rows, gu_words * 4, 32, 16,
                            CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = tensor_map_2d(&gus, dt, c.gus, gu_groups, gu_rows, gu_groups * 2, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    if ((rc = tensor_map_2d(&gub, dt, c.gub, gu_groups, gu_rows, gu_groups * 2, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    if ((rc = tensor_map_2d(&dnw, CU_TENSOR_MAP_DATA_TYPE_UINT32, c.dnw, dn_words, dn_rows, dn_words * 4, 32, 16,
                            CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = tensor_map_2d(&dns, dt, c.dns, dn_groups, dn_rows, dn_groups * 2, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    if ((rc = tensor_map_2d(&dnb, dt, c.dnb, dn_groups, dn_rows, dn_groups * 2, 8, 16, CU_TENSOR_MAP_SWIZZLE_NONE)))
        return rc;
    qmm::MdArgs a{};
    a.x = static_cast<const uint16_t*>(c.x);
    a.ids = c.ids;
    a.wts = c.wts;
    a.y = static_cast<uint16_t*>(c.y);
    a.ctr = static_cast<unsigned long long*>(c.ws);
    a.h = reinterpret_cast<uint16_t*>(static_cast<char*>(c.ws) + 256);
    a.T = c.T;
    a.top_k = c.top_k;
    a.E = c.E;
    a.H = c.H;
    a.I = c.I;
    a.UA = P * (c.I / 8);
    a.UB = c.T * (c.H / 16);
    // K slices per phase-A unit: while one slice per unit leaves a CTA with
    // fewer items than warps, halve the slices (up to 4 per unit), so that
    // every item of a small launch has a warp of its own
    {
        using R1 = qmm::QRing<BITS, GS, 1, qmm::kMdStages>;
        const int SA = c.H / (R1::CPS * qmm::QGeom<BITS, GS>::CH);
        const int units_per_cta = (a.UA + sms - 1) / sms;
        int ks = 1;
        while (ks < 4 && units_per_cta * ks * 2 <= qmm::kMdWarps && SA % (ks * 2) == 0) ks *= 2;
        a.KS = ks;
    }
    // A plain launch: the expert ids and router weights come from work this
    // library does not own (a router's top-k, or an exchange's join), the
    // case in which the MoE glue kernels take no programmatic launch.  The
    // kernel still lets its own dependents start early.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)sms, 1, 1);  // the barrier's arrival count: fixed per device
    cfg.blockDim = dim3(32 * qmm::kMdWarps, 1, 1);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = c.st;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, guw, gus, gub, dnw, dns, dnb, a);
    if (e != cudaSuccess) cudaGetLastError();
    return cuda_status(e, "moe_glu_decode launch");
}

template <int BITS, int GS>
static int launch_md_dt(const MoeDecodeCall& c) {
    return c.dtype == QMM_F16 ? launch_md_t<BITS, GS, true>(c) : launch_md_t<BITS, GS, false>(c);
}

template <int BITS>
static int launch_md_gs(const MoeDecodeCall& c) {
    switch (c.gs) {
        case 32: return launch_md_dt<BITS, 32>(c);
        case 64: return launch_md_dt<BITS, 64>(c);
        case 128: return launch_md_dt<BITS, 128>(c);
    }
    set_error("moe_glu_decode: group_size=%d unsupported", c.gs);
    return QMM_EUNSUPPORTED;
}

int launch_moe_glu_decode(const MoeDecodeCall& c) {
    return c.bits == 8 ? launch_md_gs<8>(c) : launch_md_gs<4>(c);
}

}  // namespace qmm_host
