// qmv_sk.cu -- persistent stream-K decode / verify kernel for M <= 16 rows
// per weight tile: dense quantized matmul, and the expert-gathered form.
//
// Same per-chunk arithmetic as qmv.cu (qmv_chunk.cuh), different schedule:
// the (row tile, K stage) units of the whole problem are laid out tile-major
// and a FIXED number of warps each takes an equal, contiguous range of them.
// Every SM therefore gets the same amount of weight stream regardless of how
// the row tiles divide by 148 SMs (the wave quantisation that idles most SMs
// for 160- or 192-tile matrices).
//
// A tile whose units span several warps is summed through a small workspace:
// each warp writes its partial to one of its two slots (a contiguous range of
// units has a partial tile at most at each end), and whichever warp finishes
// the tile last adds the owners' partials in owner (= K) order and stores y.
// The segment boundaries depend on the problem shape only, so an M-row call
// reduces every row in exactly the order of a single-row call, and the result
// is identical from run to run.  Counters return to zero after every tile.
//
// Dense: tile t covers weight rows [t*ROWS, (t+1)*ROWS) and all M rows of x.
// Gather: the rows are sorted by expert and cut into items of at most 8*MT
// rows of one expert; tile (item, j) covers rows [j*ROWS, (j+1)*ROWS) of that
// expert's matrix (one TMA map over the stacked [E*N] rows) and the item's x
// rows (row_src), and stores to the item's sorted rows (or row_dst, scaled
// by row_scale).  The item count is device data, so the unit split is made
// after griddepcontrol.wait.
//
// Weights stream through a per-warp TMA ring (16*RW rows x 128 B stages).
// The kernel is launched with programmatic stream serialization: in the dense
// form it streams its first weight stages before griddepcontrol.wait,
// overlapping the previous kernel's tail.

#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "tc.cuh"
#include "tma.cuh"
#include "qmv_chunk.cuh"

namespace qmm {

struct SkArgs {
    const uint16_t* x;
    const uint16_t* sc;
    const uint16_t* bi;
    uint16_t* y;
    int M, N, K;
    int Ut;             // K stages per tile
    int T;              // dense: row tiles of 16*RW rows
    int warps_total;    // warps launched (the split uses min(warps_total, units))
    float* slots;       // [warps_total][2][32 * RW * 2 * 4]
    int* counters;      // [tiles], zero between calls
    // gather
    const int4* item_info;     // [items]: (expert, first sorted row, rows, 0)
    const int32_t* n_items;    // device count of items
    const uint32_t* row_src;   // x row of sorted row s, or null (s)
    const uint32_t* row_dst;   // output row of sorted row s, or null (s)
    const float* row_scale;    // output scale of sorted row s, or null
    int TN;                    // row tiles per expert
    int x_rows, y_rows;        // bounds: rows outside read zeros / are not stored
    long long x_stride;        // gather: elements from one x row to the next (>= K)
    int glu;                   // 1: rows interleave gate/up per 16-row block; store silu(gate)*up, N/2 columns
};


QMM_DEVINL int unit_owner(long long u, long long total, int wt) {
    return (int)(((u + 1) * wt - 1) / total);
}

// Tile counter increment with release (this warp's partial-sum stores, which
// __syncwarp ordered before it, become visible first) and acquire (the last
// warp then sees every other segment's stores).
QMM_DEVINL int atom_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Launch shape of the stream-K kernel per row-tile height (16*RW rows) and
// MMA n-tiles (MT): TMA ring stages, warps per CTA and resident CTAs per SM
// (shared memory and registers at that occupancy).
template <int RW>
constexpr int sk_stages() {
    return RW == 1 ? 3 : 2;
}
template <int RW>
constexpr int sk_wpc() {
    return RW == 4 ? 3 : 4;
}
template <int RW, int MT>
constexpr int sk_minb() {
    return RW == 4 ? 3 : ((RW == 1 && MT == 1) ? 5 : 4);
}

// STMA: scales and biases arrive with the weights through TMA (a box of 8
// groups x tile rows per stage; needs a 16-byte scale row stride) instead of
// per-chunk loads from L2.
// XT: the activation rows of each stage arrive through TMA too (a box of M
// rows x the stage's K values), read from shared memory instead of L2; used
// when M is small enough for the extra ring (M <= 4).
template <int BITS, int GS, bool F16, int MT, int RW, int MINB, bool STMA, bool XT, bool GATHER>
__global__ void __launch_bounds__(32 * sk_wpc<RW>(), MINB)
    qmv_sk_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap smap,
                  const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap xmap, SkArgs a) {
    using G_ = QGeom<BITS, GS>;
    using R_ = QRing<BITS, GS, RW, sk_stages<RW>()>;
    using H = Half<F16>;
    constexpr int WPT = G_::WPT, XR = G_::XR, STEPS = G_::STEPS, VPT = G_::VPT;
    constexpr int CH = G_::CH, CPG = G_::CPG, CPS = R_::CPS, STG = R_::STG, ROWS = R_::ROWS;
    constexpr int CBU = R_::CHUNK_BYTES / 16;
    constexpr int NV = RW * MT * 4;       // partial values per lane
    constexpr int SLOT = 32 * NV;         // floats per slot

    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned by pointer arithmetic on the __shared__ array, so every
    // pointer derived from it stays in the shared window (plain LDS, no
    // generic loads)
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int N = a.N, K = a.K, G = K / GS, C = K / CH;
    const int gw = blockIdx.x * nwarps + warp;

    constexpr int SC_BYTES = ROWS * 16;  // one 8-group box of scales (or biases) per stage
    constexpr int SV = CPS * CH;         // K values per stage
    const int XB = XT ? a.M * SV * 2 : 0;  // activation bytes per stage (M rows)
    uint8_t* sring = smem + nwarps * R_::WARP_BYTES + warp * (STG * 2 * SC_BYTES);
    uint8_t* xring = smem + nwarps * (R_::WARP_BYTES + (STMA ? STG * 2 * SC_BYTES : 0)) + warp * (STG * XB);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + nwarps * (R_::WARP_BYTES + (STMA ? STG * 2 * SC_BYTES : 0)) +
                                                 nwarps * STG * XB);
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

    // the problem's units and the warps that share them
    long long total;
    if constexpr (GATHER) {
        pdl_wait();  // the item table is written by the kernel before this one
        total = (long long)ld_dep(a.n_items) * a.TN * a.Ut;
    } else {
        total = (long long)a.T * a.Ut;
    }
    const int wt = total < a.warps_total ? (int)total : a.warps_total;
    if (gw >= wt) return;  // no unit for this warp (no barrier below spans warps)

    // this warp's contiguous unit range
    const long long ua = total * gw / wt;
    const long long ub = total * (gw + 1) / wt;
    const int nst = (int)(ub - ua);

    // first weight row of tile vt (the TMA row coordinate of weights and scales)
    auto tile_wrow = [&](int vt) {
        if constexpr (GATHER) {
            const int item = vt / a.TN;
            return ld_dep(&a.item_info[item].x) * a.N + (vt - item * a.TN) * ROWS;
        } else {
            return vt * ROWS;
        }
    };

    // (tile, K stage) of the next stage to issue, advanced one unit at a time
    int i_tile = (int)(ua / a.Ut), i_ku = (int)(ua - (long long)i_tile * a.Ut);
    int i_wrow = tile_wrow(i_tile);
    // weights (+ scales) of one stage; the barrier also expects the stage's
    // activation box, which issue_x adds
    auto issue_w = [&](int s) {
        const int wrow = i_wrow, ku = i_ku;
        if (++i_ku == a.Ut) {
            i_ku = 0;
            ++i_tile;
            if (i_tile * (long long)a.Ut < ub) i_wrow = tile_wrow(i_tile);
        }
        // the issue state above advances in every lane (warp-uniform values);
        // one elected lane issues the copies
        if (elect_one()) {
            mbar_expect_tx(bar0 + 8 * s, R_::STAGE_BYTES + (STMA ? 2 * SC_BYTES : 0) + XB);
            tma_load_2d(ring0 + s * R_::STAGE_BYTES, &wmap, bar0 + 8 * s, ku * CPS * G_::WPG, wrow);
            if constexpr (STMA) {
                // groups of this stage start at ku*CPS/CPG; the box starts at the
                // 8-group (16-byte) boundary below and the kernel indexes past it
                const int gx = (ku * (CPS / CPG)) & ~7;
                const uint32_t sdst = smem_u32(sring) + s * 2 * SC_BYTES;
                tma_load_2d(sdst, &smap, bar0 + 8 * s, gx, wrow);
                tma_load_2d(sdst + SC_BYTES, &bmap, bar0 + 8 * s, gx, wrow);
            }
        }
        __syncwarp();
        return ku;
    };
    auto issue_x = [&](int s, int ku) {
        if constexpr (XT) {
            if (elect_one()) tma_load_2d(smem_u32(xring) + s * XB, &xmap, bar0 + 8 * s, ku * SV, 0);
            __syncwarp();
        }
    };
    int pro_ku[STG];
    if (lane == 0 && nst > 0) {
        tma_prefetch_desc(&wmap);
        if constexpr (STMA) {
            tma_prefetch_desc(&smap);
            tma_prefetch_desc(&bmap);
        }
        if constexpr (XT) tma_prefetch_desc(&xmap);
    }
    // weights and scales do not depend on the previous kernel: stream them now
    for (int s = 0; s < STG && s < nst; ++s) pro_ku[s] = issue_w(s);
    if constexpr (!GATHER) pdl_wait();  // x (and y's readers) belong to the previous kernel
    if constexpr (XT) {
        for (int s = 0; s < STG && s < nst; ++s) issue_x(s, pro_ku[s]);
    }
    // activation rows: the same for every tile (dense), the tile's item's rows (gather)
    const uint16_t* xrow[MT];
    bool xv[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m = 8 * mt + g;
        xv[mt] = m < a.M;
        xrow[mt] = a.x + (long long)(xv[mt] ? m : 0) * K + t * VPT;
    }
    // current tile: first weight row, first output column, and (gather) the
    // item's first sorted row and row count
    int t_wrow = 0, t_n0 = 0, t_r0 = 0, t_cnt = a.M;
    auto enter_tile = [&](int tile) {
        t_wrow = tile_wrow(tile);
        if constexpr (GATHER) {
            const int item = tile / a.TN;
            const int4 inf = ld_dep(&a.item_info[item]);
            t_n0 = (tile - item * a.TN) * ROWS;
            t_r0 = inf.y;
            t_cnt = inf.z;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int m = 8 * mt + g;
                uint32_t src = 0;
                bool ok = m < t_cnt;
                if (ok) {
                    src = a.row_src ? ld_dep(a.row_src + t_r0 + m) : (uint32_t)(t_r0 + m);
                    ok = src < (uint32_t)a.x_rows;  // a row outside x reads zeros
                }
                xv[mt] = ok;
                xrow[mt] = a.x + (long long)(ok ? src : 0) * a.x_stride + t * VPT;
            }
        } else {
            t_n0 = tile * ROWS;
        }
    };
    const uint32_t tb = (uint32_t)t * WPT * 4;
    const uint32_t tconst = ((((tb >> 4) ^ (uint32_t)g) & (CBU - 1)) << 4) | (tb & 15);
    const uint32_t hkey = (uint32_t)g & 7u & ~(uint32_t)(CBU - 1);
    const uint32_t rowbase = (uint32_t)g * 128;

    float res[RW][MT][4];
    int cur_tile = -1, seg_k0 = 0;

    // write the finished (or partial) tile
    auto flush = [&](int tile, int k0, int k1) {
        const bool whole = (k0 == 0 && k1 == a.Ut);
        float out[RW][MT][4];
        bool store = whole;
        if (!whole) {
            const long long u0 = (long long)tile * a.Ut;
            const int f = unit_owner(u0, total, wt);
            const int l = unit_owner(u0 + a.Ut - 1, total, wt);
            // warp w's slot for this tile: 0 if w's range starts inside the tile
            // (every owner after the first does), 1 if it started before it
            const bool f_before = total * f / wt < u0;
            auto slot_of = [&](int w) {
                return a.slots + ((long long)w * 2 + (w == f && f_before ? 1 : 0)) * SLOT + lane * NV;
            };
            float4* mine = reinterpret_cast<float4*>(slot_of(gw));
#pragma unroll
            for (int v = 0; v < NV / 4; ++v) {
                const int i0 = 4 * v;
                const float* rr = &res[0][0][0];
                mine[v] = make_float4(rr[i0], rr[i0 + 1], rr[i0 + 2], rr[i0 + 3]);
            }
            __syncwarp();  // every lane's slot stores precede lane 0's release
            int prev = 0;
            if (lane == 0) prev = atom_add_acq_rel(a.counters + tile, 1);
            prev = __shfl_sync(0xffffffffu, prev, 0);
            __syncwarp();  // lane 0's acquire precedes every lane's slot reads
            if (prev == l - f) {
                float* oo = &out[0][0][0];
#pragma unroll
                for (int i = 0; i < NV; ++i) oo[i] = 0.0f;
                // every owner's partial (this warp's own included: it was
                // stored above) in owner order; loads issued four owners at a
                // time so their L2 latencies overlap
                constexpr int QB = 4, NQ = NV / 4;
                int sg = f;
                for (; sg + QB <= l + 1; sg += QB) {
                    float4 q[QB][NQ];
#pragma unroll
                    for (int b = 0; b < QB; ++b) {
                        const float4* pb = reinterpret_cast<const float4*>(slot_of(sg + b));
#pragma unroll
                        for (int v = 0; v < NQ; ++v) q[b][v] = __ldcg(pb + v);
                    }
#pragma unroll
                    for (int b = 0; b < QB; ++b)
#pragma unroll
                        for (int v = 0; v < NQ; ++v) {
                            oo[4 * v] += q[b][v].x;
                            oo[4 * v + 1] += q[b][v].y;
                            oo[4 * v + 2] += q[b][v].z;
                            oo[4 * v + 3] += q[b][v].w;
                        }
                }
                for (; sg <= l; ++sg)
#pragma unroll
                    for (int v = 0; v < NQ; ++v) {
                        const float4 q = __ldcg(reinterpret_cast<const float4*>(slot_of(sg)) + v);
                        oo[4 * v] += q.x;
                        oo[4 * v + 1] += q.y;
                        oo[4 * v + 2] += q.z;
                        oo[4 * v + 3] += q.w;
                    }
                if (lane == 0) a.counters[tile] = 0;
                store = true;
            }
        } else {
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int c = 0; c < 4; ++c) out[r][mt][c] = res[r][mt][c];
        }
        if (store) {
            // output row and scale of each of this lane's activation rows
            long long orow[MT][2];
            float oscale[MT][2];
            bool oval[MT][2];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int c1 = 0; c1 < 2; ++c1) {
                    const int m = 8 * mt + 2 * t + c1;
                    oval[mt][c1] = m < t_cnt;
                    orow[mt][c1] = m;
                    oscale[mt][c1] = 1.0f;
                    if constexpr (GATHER) {
                        if (oval[mt][c1]) {
                            const uint32_t d = a.row_dst ? ld_dep(a.row_dst + t_r0 + m) : (uint32_t)(t_r0 + m);
                            oval[mt][c1] = d < (uint32_t)a.y_rows;  // a row outside y is not stored
                            orow[mt][c1] = d;
                            if (a.row_scale) oscale[mt][c1] = ld_dep(a.row_scale + t_r0 + m);
                        }
                    }
                }
            if (GATHER && a.glu) {
                // rows 16b..16b+7 of each 16-row block are gate rows of channels
                // 8b..8b+7, rows 16b+8.. the matching up rows: this lane holds
                // both values of channel 8b+g
                const int NO = N / 2;
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int c1 = 0; c1 < 2; ++c1) {
                            const int ch = t_n0 / 2 + 8 * r + g;
                            if (ch < NO && oval[mt][c1]) {
                                const float gt = out[r][mt][c1], up = out[r][mt][2 + c1];
                                const float v = gt / (1.0f + expf(-gt)) * up * oscale[mt][c1];
                                a.y[orow[mt][c1] * NO + ch] = H::from_f32(v);
                            }
                        }
            } else {
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            const int n = t_n0 + 16 * r + g + 8 * (c >> 1);
                            const int c1 = c & 1;
                            if (n < N && oval[mt][c1]) {
                                const float v = GATHER ? out[r][mt][c] * oscale[mt][c1] : out[r][mt][c];
                                a.y[orow[mt][c1] * N + n] = H::from_f32(v);
                            }
                        }
            }
        }
    };

    // Activations, scales and biases one chunk ahead, double-buffered by chunk
    // parity (chunk c of a stage uses buffer c & 1; CPS is even, so chunk 0 of
    // the next stage lands in buffer 0 again): no register copies.  Addresses
    // are per-stage bases plus compile-time offsets.
    uint32_t xb[2][MT][XR];
    uint16_t sb[2][RW][2], bb[2][RW][2];
    uint32_t sbw[RW][2][2];  // (scale, bias) pairs of two groups, through TMA
    const uint16_t* xs_base[MT];
    const uint16_t* ss_base[RW][2];
    const uint16_t* bs_base[RW][2];
    auto stage_bases = [&](int tile, int ku) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) xs_base[mt] = xrow[mt] + ku * (CPS * CH);
        if constexpr (!STMA) {
            const int g_off = ku * (CPS / CPG);
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // rows past N read a valid row of the tile's matrix; their results are dropped
                    int n = t_n0 + 16 * r + 8 * h + g;
                    n = n < N ? n : N - 1;
                    const long long row = (long long)(t_wrow - t_n0) + n;
                    ss_base[r][h] = a.sc + row * G + g_off;
                    bs_base[r][h] = a.bi + row * G + g_off;
                }
        }
    };
    // fetch chunk `c` (0..CPS, CPS = first chunk of the next stage) into buffer B
    auto fetch = [&](int B, int c) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) load_x<XR>(xb[B][mt], xs_base[mt] + c * CH, xv[mt]);
        if constexpr (!STMA) {
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    sb[B][r][h] = ldg_u16(ss_base[r][h] + c / CPG);
                    bb[B][r][h] = ldg_u16(bs_base[r][h] + c / CPG);
                }
        }
    };

    // activations of chunk `c` of stage slot `s` from the stage's TMA box
    // (rows past M read row 0: they only feed output columns that are dropped)
    auto fetch_xs = [&](int B, int s, int c) {
        if constexpr (XT) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int m = 8 * mt + g < a.M ? 8 * mt + g : 0;
                const uint32_t addr = smem_u32(xring) + s * XB + (uint32_t)((m * SV + c * CH + t * VPT) * 2);
#pragma unroll
                for (int i = 0; i < XR; i += 4)
                    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(xb[B][mt][i]), "=r"(xb[B][mt][i + 1]), "=r"(xb[B][mt][i + 2]),
                                   "=r"(xb[B][mt][i + 3])
                                 : "r"(addr + 4 * i));  // register i holds values 2i, 2i+1
            }
        }
    };

    int m_tile = (int)(ua / a.Ut), m_ku = (int)(ua - (long long)m_tile * a.Ut);
    for (int st = 0; st < nst; ++st) {
        const int tile = m_tile, ku = m_ku;
        if (++m_ku == a.Ut) {
            m_ku = 0;
            ++m_tile;
        }
        if (tile != cur_tile) {
            cur_tile = tile;
            seg_k0 = ku;
            enter_tile(tile);
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int c = 0; c < 4; ++c) res[r][mt][c] = 0.0f;
            stage_bases(tile, ku);
            if constexpr (!XT) fetch(0, 0);
        }
        // whether this stage's last chunk prefetches the next stage's first chunk
        const bool next_same_tile = (ku + 1 < a.Ut) && (st + 1 < nst);
        const int s = st % STG;
        mbar_wait_bounded(bar0 + 8 * s, (uint32_t)(st / STG) & 1u, abort, &g_qmv_error);
        if constexpr (XT) fetch_xs(0, s, 0);
        const uint32_t stage_addr = ring0 + s * R_::STAGE_BYTES + rowbase;
        const bool full = (ku + 1) * CPS <= C;
        // FULL: every chunk of the stage lies inside K (no per-chunk checks)
        auto do_chunk = [&](auto cc, auto fullc) {
            constexpr int c = decltype(cc)::value;
            constexpr bool FULL = decltype(fullc)::value;
            constexpr int B = c & 1;
            if constexpr (XT) {
                if constexpr (c + 1 < CPS) {
                    if (FULL || ku * CPS + c + 1 < C) fetch_xs(B ^ 1, s, c + 1);
                }
            } else if constexpr (c + 1 < CPS) {
                if (FULL || ku * CPS + c + 1 < C) fetch(B ^ 1, c + 1);
            } else {
                if (next_same_tile) fetch(B ^ 1, CPS);
            }
            float s_[RW][2], b_[RW][2];
            if constexpr (STMA) {
                // this chunk's group inside the stage's 8-group box
                constexpr int GPS = CPS / CPG, gq = c / CPG;
                const int gi = ((ku * GPS) & 7) + gq;
                const uint16_t* sp = reinterpret_cast<const uint16_t*>(sring + s * 2 * SC_BYTES) + g * 8;
                if constexpr (GPS % 2 == 0) {
                    // an even number of groups per stage: read (scale, bias)
                    // words for two groups at a time (gi is even when gq is)
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
            } else {
#pragma unroll
                for (int r = 0; r < RW; ++r)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        s_[r][h] = H::to_f32(sb[B][r][h]);
                        b_[r][h] = H::to_f32(bb[B][r][h]);
                    }
            }
            uint32_t wv[RW][2][WPT];
            const uint32_t cofs = (((((uint32_t)(c * CBU)) ^ hkey) & 7u) << 4) | tconst;
            lds_tile_rows<RW, WPT>(stage_addr + cofs, wv);
            chunk_math<BITS, F16, MT, RW, XR, WPT, STEPS>(res, xb[B], wv, s_, b_);
        };
        if (full) {
            unroll_chunks<CPS>([&](auto cc) { do_chunk(cc, std::true_type{}); });
        } else {
            unroll_chunks<CPS>([&](auto cc) {
                if (ku * CPS + decltype(cc)::value < C) do_chunk(cc, std::false_type{});
            });
        }
        if (next_same_tile) stage_bases(tile, ku + 1);
        __syncwarp();
        if (st + STG < nst) issue_x(s, issue_w(s));
        if (ku == a.Ut - 1 || st == nst - 1) flush(tile, seg_k0, ku + 1);
    }
}

}  // namespace qmm

namespace qmm_host {

using qmm::SkArgs;

// Fixed schedule of the stream-K kernel for an (N, K) matrix.  Nothing here
// depends on M.
struct SkPlan {
    int rw, T, Ut, warps_total;
};

static int sk_stages_per_row(long long K, int gs, int bits) {
    const int ch = gs < 64 ? gs : 64;
    const int cps = 128 / (ch * bits / 8);
    return (int)((K / ch + cps - 1) / cps);
}

// M <= 8 calls (one MMA n-tile) share one plan, so each of their rows has the
// bits of a single-row call; M = 9..16 use 16-row tiles (register budget).
static int sk_wpc_rt(int rw) { return rw == 4 ? qmm::sk_wpc<4>() : qmm::sk_wpc<1>(); }
static int sk_minb_rt(int rw, int mt) {
    return rw == 4 ? qmm::sk_minb<4, 1>() : (rw == 1 && mt == 1 ? qmm::sk_minb<1, 1>() : qmm::sk_minb<2, 1>());
}

static SkPlan sk_plan(long long N, long long K, int gs, int bits, int mt) {
    SkPlan p;
    p.rw = mt == 1 ? 2 : 1;  // 32-row tiles for M <= 8 (measured faster at every layer shape)
    p.T = (int)((N + 16 * p.rw - 1) / (16 * p.rw));
    p.Ut = sk_stages_per_row(K, gs, bits);
    const long long total = (long long)p.T * p.Ut;
    // resident CTAs per SM; never more warps than units, so every warp owns
    // at least one unit (a tile's segments are then consecutive warps)
    const int wpc = sk_wpc_rt(p.rw);
    const int ctas = sk_minb_rt(p.rw, mt);
    long long wt = 148LL * wpc * ctas;
    if (wt > total) wt = total >= wpc ? total / wpc * wpc : total;
    p.warps_total = (int)wt;
    return p;
}

// Workspace layout, the same for every shape so that calls of different
// shapes (dense and gathered) can share one buffer: a fixed block of
// kSkCounters tile counters (zero between calls), then two partial-sum slots
// per launched warp (no invariant).  A slot holds 32 lanes x RW*MT*4 floats,
// at most 1 KiB (RW*MT <= 2).
constexpr long long kSkCounters = 65536;
constexpr size_t kSkCounterBytes = kSkCounters * sizeof(int);
// The gathered form counts (item, row tile) pairs, whose bound grows with the
// rows (padding rows of an expert-parallel exchange included): 1 MiB of them.
constexpr long long kSkGatherCounters = 262144;
constexpr size_t kSkGatherCounterBytes = kSkGatherCounters * sizeof(int);
constexpr int kSkMaxWarps = 148 * 4 * 5;
constexpr size_t kSkSlotBytes = 1024;  // RW*MT <= 2 (64-row tiles use 2 KiB slots, with fewer warps)

// The counter block, then two slots per launched warp.
size_t sk_workspace(long long M, long long N, long long K, int gs, int bits) {
    const int mt = M <= 8 ? 1 : 2;
    const SkPlan p = sk_plan(N, K, gs, bits, mt);
    return kSkCounterBytes + (size_t)p.warps_total * 2 * (512 * (size_t)p.rw * mt);
}

// The gathered form's slots are sized for the most warps any launch uses, so
// the size depends on nothing but the counter block.
size_t sk_gather_workspace() { return kSkGatherCounterBytes + (size_t)kSkMaxWarps * 2 * kSkSlotBytes; }

// Whether the activation ring (M rows per stage) fits beside the weight and
// scale rings with the register-limited number of resident CTAs per SM.
template <int BITS, int GS, int RW>
static bool sk_xt_fits(int M) {
    using R_ = qmm::QRing<BITS, GS, RW, qmm::sk_stages<RW>()>;
    using G_ = qmm::QGeom<BITS, GS>;
    constexpr int MINB = qmm::sk_minb<RW, 1>();
    const size_t per_warp = (size_t)R_::WARP_BYTES + (size_t)R_::STG * 2 * R_::ROWS * 16 +
                            (size_t)R_::STG * M * R_::CPS * G_::CH * 2 + R_::STG * 8 + 4;
    const size_t per_cta = qmm::sk_wpc<RW>() * per_warp + 1024 + 1024;  // + alignment slack + runtime reservation
    return MINB * per_cta <= 228 * 1024;
}

// w_rows: rows of the weight map (N dense, E*N gathered: the experts' matrices stacked)
template <int BITS, int GS, bool F16, int MT, int RW, bool STMA, bool XT, bool GATHER>
static int launch_sk_t(const SkArgs& a, const uint32_t* w, long long w_rows, cudaStream_t st) {
    using R_ = qmm::QRing<BITS, GS, RW, qmm::sk_stages<RW>()>;
    using G_ = qmm::QGeom<BITS, GS>;
    constexpr int MINB = qmm::sk_minb<RW, MT>();  // resident CTAs per SM (register / shared-memory budget)
    constexpr int WPC = qmm::sk_wpc<RW>();
    auto kern = qmm::qmv_sk_kernel<BITS, GS, F16, MT, RW, MINB, STMA, XT, GATHER>;
    const int W = a.warps_total < WPC ? a.warps_total : WPC;
    constexpr int SV = R_::CPS * G_::CH;
    constexpr size_t SC = STMA ? (size_t)R_::STG * 2 * R_::ROWS * 16 : 0;
    const size_t XS = XT ? (size_t)R_::STG * a.M * SV * 2 : 0;
    auto smem_for = [&](int w_, size_t xs) {
        return (size_t)w_ * (R_::WARP_BYTES + SC + xs) + w_ * R_::STG * 8 + w_ * 4 + 1024;
    };
    const size_t smem = smem_for(W, XS);
    {
        // the largest request: four warps and, with XT, the most activation rows that fit
        int mmax = 0;
        if (XT)
            for (int m = 1; m <= 8; ++m)
                if (sk_xt_fits<BITS, GS, RW>(m)) mmax = m;
        const size_t xmax = (size_t)R_::STG * mmax * SV * 2;
        const int rc0 = ensure_smem_limit((const void*)kern, (int)smem_for(WPC, xmax), "qmv_sk smem attribute");
        if (rc0) return rc0;
    }
    CUtensorMap wmap, smap, bmap, xmap;
    const uint64_t wrow = (uint64_t)a.K * BITS / 32;
    int rc = tensor_map_2d(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, wrow, (uint64_t)w_rows, wrow * 4, 32,
                           (uint32_t)R_::ROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if constexpr (STMA) {
        const uint64_t G = (uint64_t)a.K / GS;
        const CUtensorMapDataType dt = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        rc = tensor_map_2d(&smap, dt, a.sc, G, (uint64_t)w_rows, G * 2, 8, (uint32_t)R_::ROWS,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
        rc = tensor_map_2d(&bmap, dt, a.bi, G, (uint64_t)w_rows, G * 2, 8, (uint32_t)R_::ROWS,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    } else {
        smap = wmap;
        bmap = wmap;
    }
    if constexpr (XT) {
        const CUtensorMapDataType dt = F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
        rc = tensor_map_2d(&xmap, dt, a.x, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)a.K * 2, SV, (uint32_t)a.M,
                           CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    } else {
        xmap = wmap;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(a.warps_total / W), 1, 1);
    cfg.blockDim = dim3(32 * W, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wmap, smap, bmap, xmap, a);
    if (e != cudaSuccess) cudaGetLastError();
    return cuda_status(e, "qmv_sk launch");
}

template <int BITS, int GS, bool F16, bool STMA, bool GATHER>
static int launch_sk_s(const SkArgs& a, const uint32_t* w, long long w_rows, int mt, int rw, cudaStream_t st) {
    if (mt == 1) {
        if (!GATHER && rw == 4) {  // 64-row tiles (dense only)
            if (STMA && sk_xt_fits<BITS, GS, 4>(a.M))
                return launch_sk_t<BITS, GS, F16, 1, 4, STMA, STMA, false>(a, w, w_rows, st);
            return launch_sk_t<BITS, GS, F16, 1, 4, STMA, false, false>(a, w, w_rows, st);
        }
        // dense: activations through TMA while their ring fits (small M)
        if (!GATHER && STMA && (rw == 1 ? sk_xt_fits<BITS, GS, 1>(a.M) : sk_xt_fits<BITS, GS, 2>(a.M)))
            return rw == 1 ? launch_sk_t<BITS, GS, F16, 1, 1, STMA, STMA && !GATHER, GATHER>(a, w, w_rows, st)
                           : launch_sk_t<BITS, GS, F16, 1, 2, STMA, STMA && !GATHER, GATHER>(a, w, w_rows, st);
        return rw == 1 ? launch_sk_t<BITS, GS, F16, 1, 1, STMA, false, GATHER>(a, w, w_rows, st)
                       : launch_sk_t<BITS, GS, F16, 1, 2, STMA, false, GATHER>(a, w, w_rows, st);
    }
    (void)rw;  // 16 rows per tile always use 16-row weight tiles
    return launch_sk_t<BITS, GS, F16, 2, 1, STMA, false, GATHER>(a, w, w_rows, st);
}

template <int BITS, int GS, bool F16, bool GATHER>
static int launch_sk_b(const SkArgs& a, const uint32_t* w, long long w_rows, int mt, int rw, cudaStream_t st) {
    // scales/biases through TMA need 16-byte scale rows and 16-byte aligned bases
    const bool stma = ((a.K / GS) % 8 == 0) && ((uintptr_t)a.sc % 16 == 0) && ((uintptr_t)a.bi % 16 == 0);
    return stma ? launch_sk_s<BITS, GS, F16, true, GATHER>(a, w, w_rows, mt, rw, st)
                : launch_sk_s<BITS, GS, F16, false, GATHER>(a, w, w_rows, mt, rw, st);
}

template <bool GATHER>
static int launch_sk_any(const SkArgs& a, const uint32_t* w, long long w_rows, int bits, int gs, bool f16, int mt,
                         int rw, cudaStream_t st) {
#define QMM_SK_CASE(B, S)                                                                                  \
    if (bits == B && gs == S)                                                                               \
        return f16 ? launch_sk_b<B, S, true, GATHER>(a, w, w_rows, mt, rw, st)                              \
                   : launch_sk_b<B, S, false, GATHER>(a, w, w_rows, mt, rw, st);
    QMM_SK_CASE(4, 32)
    QMM_SK_CASE(4, 64)
    QMM_SK_CASE(4, 128)
    QMM_SK_CASE(8, 32)
    QMM_SK_CASE(8, 64)
    QMM_SK_CASE(8, 128)
#undef QMM_SK_CASE
    set_error("qmv: bits=%d group_size=%d not supported", bits, gs);
    return QMM_EUNSUPPORTED;
}

int launch_qmv_sk(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st) {
    const int mt = M <= 8 ? 1 : 2;
    const SkPlan p = sk_plan(N, K, gs, bits, mt);
    if (p.T > kSkCounters) {
        set_error("qmv: N=%d needs %d row tiles (limit %lld)", N, p.T, kSkCounters);
        return QMM_EUNSUPPORTED;
    }
    if (ws_bytes < sk_workspace(M, N, K, gs, bits)) {
        set_error("qmv: workspace %zu < %zu bytes", ws_bytes, sk_workspace(M, N, K, gs, bits));
        return QMM_EINVAL;
    }
    SkArgs a{};
    a.x = x;
    a.sc = sc;
    a.bi = bi;
    a.y = y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.T = p.T;
    a.Ut = p.Ut;
    a.warps_total = p.warps_total;
    char* wsb = static_cast<char*>(ws);
    a.counters = reinterpret_cast<int*>(wsb);
    a.slots = reinterpret_cast<float*>(wsb + kSkCounterBytes);
    return launch_sk_any<false>(a, w, N, bits, gs, f16, mt, p.rw, st);
}

// Rows per gather item (8 or 16) for `rows` sorted rows over E experts:
// 16-row items (two MMA n-tiles) once the experts average 8 rows or more.
int sk_gather_item_rows(long long rows, long long E) { return rows >= 8 * E ? 16 : 8; }

// Upper bound of the item count, from host-known sizes only.
long long sk_gather_items_max(long long rows, long long E) {
    const int ir = sk_gather_item_rows(rows, E);
    return rows / ir + (E < rows ? E : rows);
}

// Whether the stream-K gather can take this problem (tile counters).
bool sk_gather_fits(long long rows, long long E, long long N) {
    const int rw = sk_gather_item_rows(rows, E) == 8 ? 2 : 1;
    return sk_gather_items_max(rows, E) * ((N + 16 * rw - 1) / (16 * rw)) <= kSkGatherCounters;
}

// Gathered form over expert-sorted rows.  item_info / n_items come from the
// segment-table kernel (items of sk_gather_item_rows(rows, E) rows).  ws holds
// sk_gather_workspace() bytes, its counter block zero.
int launch_qmv_sk_gather(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                         const int4* item_info, const int32_t* n_items, const uint32_t* row_src,
                         const uint32_t* row_dst, const float* row_scale, long long rows, long long x_rows,
                         long long E, int N, int K, int gs, int bits, bool f16, void* ws, cudaStream_t st, int glu,
                         long long x_stride) {
    const int ir = sk_gather_item_rows(rows, E);
    const int mt = ir / 8, rw = mt == 1 ? 2 : 1;
    const int TN = (N + 16 * rw - 1) / (16 * rw);
    const int Ut = sk_stages_per_row(K, gs, bits);
    const long long units_max = sk_gather_items_max(rows, E) * TN * Ut;
    long long wt = 148LL * 4 * 4;
    if (wt > units_max) wt = units_max >= 4 ? units_max / 4 * 4 : units_max;
    SkArgs a{};
    a.x = x;
    a.sc = sc;
    a.bi = bi;
    a.y = y;
    a.M = ir;
    a.N = N;
    a.K = K;
    a.Ut = Ut;
    a.warps_total = (int)wt;
    char* wsb = static_cast<char*>(ws);
    a.counters = reinterpret_cast<int*>(wsb);
    a.slots = reinterpret_cast<float*>(wsb + kSkGatherCounterBytes);
    a.item_info = item_info;
    a.n_items = n_items;
    a.row_src = row_src;
    a.row_dst = row_dst;
    a.row_scale = row_scale;
    a.TN = TN;
    a.x_rows = (int)x_rows;
    a.x_stride = x_stride > 0 ? x_stride : K;
    a.y_rows = (int)rows;
    a.glu = glu;
    return launch_sk_any<true>(a, w, E * (long long)N, bits, gs, f16, mt, rw, st);
}

int qmv_sk_device_error(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, qmm::g_qmv_error, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        const int z = 0;
        cudaMemcpyToSymbol(qmm::g_qmv_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace qmm_host
