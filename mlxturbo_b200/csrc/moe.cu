// moe.cu -- MoE glue kernels on the device, sm_100a: segment tables,
// deterministic counting sort, combine, and elementwise dequantisation.
//
//  * segment tables   <- mlxturbo/kernels/moe_grouped_gemm.py:818-855
//                        (counts_from_sorted_ids, segment_tables)
//  * counting sort    <- mlxturbo/kernels/moe_counting_sort.py:41-80 (hist ->
//                        exclusive scan -> in-order scatter, no atomics in the
//                        output order) and _vendor/qwen4_exp.py:1775-1778
//  * combine          <- mlxturbo/kernels/moe_combine.py:1-60
// All are HBM/latency bound integer or streaming work; none uses tensor cores.

#include "common.cuh"
#include "tma.cuh"

namespace qmm {

// Block-wide exclusive scan of three counters at once (1024 threads): each
// thread passes its run's totals and gets the sum over the threads before it.
QMM_DEVINL void block_exclusive_scan3(int& a, int& b, int& c) {
    __shared__ int ws[3][32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int ia = a, ib = b, ic = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int ua = __shfl_up_sync(0xffffffffu, ia, o);
        const int ub = __shfl_up_sync(0xffffffffu, ib, o);
        const int uc = __shfl_up_sync(0xffffffffu, ic, o);
        if (lane >= o) {
            ia += ua;
            ib += ub;
            ic += uc;
        }
    }
    if (lane == 31) {
        ws[0][wid] = ia;
        ws[1][wid] = ib;
        ws[2][wid] = ic;
    }
    __syncthreads();
    if (wid == 0) {
        int va = lane < nw ? ws[0][lane] : 0, vb = lane < nw ? ws[1][lane] : 0, vc = lane < nw ? ws[2][lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int ua = __shfl_up_sync(0xffffffffu, va, o);
            const int ub = __shfl_up_sync(0xffffffffu, vb, o);
            const int uc = __shfl_up_sync(0xffffffffu, vc, o);
            if (lane >= o) {
                va += ua;
                vb += ub;
                vc += uc;
            }
        }
        ws[0][lane] = va;
        ws[1][lane] = vb;
        ws[2][lane] = vc;
    }
    __syncthreads();
    const int pa = wid ? ws[0][wid - 1] : 0, pb = wid ? ws[1][wid - 1] : 0, pc = wid ? ws[2][wid - 1] : 0;
    a = pa + ia - a;
    b = pb + ib - b;
    c = pc + ic - c;
}

// Items of at most `ir` rows of one expert, as (expert, first sorted row,
// rows, 0), for experts [e0, e1) whose rows start at `rs` and items at `ip`.
QMM_DEVINL void write_items(int4* item_info, const int32_t* counts, int e0, int e1, int rs, int ip, int ir) {
    for (int e = e0; e < e1; ++e) {
        const int c = counts[e];
        for (int r = 0; r < c; r += ir) item_info[ip++] = make_int4(e, rs + r, min(ir, c - r), 0);
        rs += c;
    }
}

// Row counts per expert (ids may be unsorted; out-of-range ids are
// ignored), then the exclusive prefixes over experts of rows, bm-row tiles
// and ir-row items, and (item_info) the items themselves.  One CTA of 1024
// threads; each thread owns a run of consecutive experts, and one block scan
// combines the runs.
// counts_in != null: take the counts as given instead of counting ids.
__global__ void segment_tables_kernel(const int32_t* __restrict__ ids, int M, const int32_t* __restrict__ counts_in,
                                      int E, int bm, int mix, int32_t* counts_out, int32_t* row_start,
                                      int32_t* tile_prefix, int32_t* item_prefix, int ir, int4* item_info) {
    extern __shared__ int32_t sh[];  // counts[E]
    for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = counts_in ? counts_in[e] : 0;
    __syncthreads();
    if (!counts_in)
        for (int i = threadIdx.x; i < M; i += blockDim.x) {
            const int e = ids[i];
            if (e >= 0 && e < E) atomicAdd(&sh[e], 1);
        }
    __syncthreads();
    const int per = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = min(E, (int)threadIdx.x * per), e1 = min(E, e0 + per);
    auto tile_rows = [&](int c) { return mix > 0 ? (c < mix ? 16 : 32) : bm; };
    int rs = 0, tp = 0, ip = 0;
    for (int e = e0; e < e1; ++e) {
        const int c = sh[e];
        rs += c;
        tp += (c + tile_rows(c) - 1) / tile_rows(c);
        ip += (c + ir - 1) / ir;
    }
    block_exclusive_scan3(rs, tp, ip);
    if (item_info) write_items(item_info, sh, e0, e1, rs, ip, ir);
    for (int e = e0; e < e1; ++e) {
        const int c = sh[e];
        if (row_start) row_start[e] = rs;
        if (tile_prefix) tile_prefix[e] = tp;
        if (item_prefix) item_prefix[e] = ip;
        rs += c;
        tp += (c + tile_rows(c) - 1) / tile_rows(c);
        ip += (c + ir - 1) / ir;
    }
    if (e0 < E && e1 == E) {  // the thread that owns the last expert writes the totals
        if (row_start) row_start[E] = rs;
        if (tile_prefix) tile_prefix[E] = tp;
        if (item_prefix) item_prefix[E] = ip;
    }
    if (counts_out)
        for (int e = threadIdx.x; e < E; e += blockDim.x) counts_out[e] = sh[e];
}

// ir-row item prefix (and items) from row_start, for qmm_segmented with the
// caller's tables: one CTA of 1024 threads, runs of experts per thread, one
// block scan.
__global__ void item_prefix_from_row_start_kernel(const int32_t* __restrict__ row_start, int E, int32_t* item_prefix,
                                                  int ir, int4* item_info) {
    const int per = (E + blockDim.x - 1) / blockDim.x;
    const int e0 = min(E, (int)threadIdx.x * per), e1 = min(E, e0 + per);
    int ip = 0, z0 = 0, z1 = 0;
    for (int e = e0; e < e1; ++e) ip += (row_start[e + 1] - row_start[e] + ir - 1) / ir;
    block_exclusive_scan3(ip, z0, z1);
    const int ip0 = ip;
    for (int e = e0; e < e1; ++e) {
        item_prefix[e] = ip;
        ip += (row_start[e + 1] - row_start[e] + ir - 1) / ir;
    }
    if (e0 < E && e1 == E) item_prefix[E] = ip;
    if (item_info) {
        ip = ip0;
        for (int e = e0; e < e1; ++e) {
            const int rs = row_start[e], c = row_start[e + 1] - rs;
            for (int r = 0; r < c; r += ir) item_info[ip++] = make_int4(e, rs + r, min(ir, c - r), 0);
        }
    }
}

// ---- deterministic stable counting sort ------------------------------------
constexpr int kSortBlock = 256;  // elements per block

// hist[e * B + b] = #{ i in block b : ids[i] == e }
// Buckets 0..E-1 are the experts; every id >= E (padding rows) goes to bucket
// E, so those rows sort, in input order, after all real rows with idx_s = E,
// which the segment tables and the gather kernels ignore.
__global__ void sort_hist_kernel(const uint32_t* __restrict__ ids, int M, int E, int B, int32_t* hist) {
    extern __shared__ int32_t sh[];
    const int b = blockIdx.x;
    for (int e = threadIdx.x; e <= E; e += blockDim.x) sh[e] = 0;
    __syncthreads();
    const int i0 = b * kSortBlock, i1 = min(M, i0 + kSortBlock);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) atomicAdd(&sh[min(ids[i], (uint32_t)E)], 1);
    __syncthreads();
    for (int e = threadIdx.x; e <= E; e += blockDim.x) hist[(size_t)e * B + b] = sh[e];
}

// Exclusive scan of n ints in place, one CTA of 1024 threads.
__global__ void exclusive_scan_kernel(int32_t* data, int n) {
    __shared__ int32_t warp_sums[32];
    __shared__ int32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int base = 0; base < n; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const int v = i < n ? data[i] : 0;
        int incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += u;
        }
        if (lane == 31) warp_sums[wid] = incl;
        __syncthreads();
        if (wid == 0) {
            int ws = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, ws, o);
                if (lane >= o) ws += u;
            }
            warp_sums[lane] = ws;  // inclusive prefix of warp totals
        }
        __syncthreads();
        const int before = (wid > 0 ? warp_sums[wid - 1] : 0) + carry;
        if (i < n) data[i] = before + incl - v;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = before + incl;
        __syncthreads();
    }
}

// One warp walks its block in index order, 32 elements at a time; lanes with
// the same expert rank themselves by lane order (match_any), so the output is
// a stable sort and identical on every run.
__global__ void sort_scatter_kernel(const uint32_t* __restrict__ ids, int M, int E, int B, int top_k,
                                    const int32_t* __restrict__ offs, uint32_t* order, uint32_t* idx_s,
                                    uint32_t* row_src, uint32_t* inv) {
    extern __shared__ int32_t cur[];  // [E+1] next free slot of each bucket for this block
    __shared__ uint32_t bids[kSortBlock];  // this block's ids, staged by all threads
    const int b = blockIdx.x;
    for (int e = threadIdx.x; e <= E; e += blockDim.x) cur[e] = offs[(size_t)e * B + b];
    const int i0 = b * kSortBlock, i1 = min(M, i0 + kSortBlock);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) bids[i - i0] = ids[i];
    __syncthreads();
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    for (int base = i0; base < i1; base += 32) {
        const int i = base + lane;
        const bool valid = i < i1;
        const uint32_t e = valid ? min(bids[i - i0], (uint32_t)E) : 0xffffffffu;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const unsigned lower = same & ((1u << lane) - 1u);
        const int rank = __popc(lower);
        int pos = 0;
        if (valid) pos = cur[e] + rank;
        __syncwarp();
        // the highest lane of each expert group advances the cursor
        if (valid && (same >> lane) == 1u) cur[e] += __popc(same);
        __syncwarp();
        if (valid) {
            order[pos] = (uint32_t)i;
            idx_s[pos] = e;
            row_src[pos] = (uint32_t)i / (uint32_t)top_k;
            inv[i] = (uint32_t)pos;
        }
    }
}

// ---- route: counting sort + segment tables in one launch ----------------------
// For decode / verify batches (rows <= kRouteMaxRows, E <= kRouteMaxExperts)
// the three sort launches and the segment-table launch above become one CTA
// of kRouteThreads threads with the same outputs, bit for bit:
//   order = stable argsort(ids) (ids >= E, the padding rows, last in input
//   order), idx_s = ids[order] (E for padding), row_src = order / top_k,
//   inv = argsort(order); row_start / item_prefix / item_info of the real
//   experts as segment_tables_kernel writes them (items of `ir` rows).
// Stable ranks without a serial pass: warp w takes the contiguous block
// [w * per, (w + 1) * per) of the rows and counts it per expert into its own
// shared-memory histogram row; an exclusive scan over (expert, warp) gives
// each warp's first slot per expert; each warp then scatters its block in
// order, ranking equal experts inside 32-row chunks with match_any.
// (moe_counting_sort.py:41-80 hist -> scan -> in-order scatter;
//  moe_grouped_gemm.py:818-867 row_start / tile prefix tables.)
constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;
constexpr int kRouteMaxRows = 16384;
constexpr int kRouteMaxExperts = 1024;

__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(const uint32_t* ids, int M, int E, int top_k, int ir,
                                                                  uint32_t* order, uint32_t* idx_s, uint32_t* row_src,
                                                                  uint32_t* inv, int32_t* row_start,
                                                                  int32_t* item_prefix, int4* item_info) {
    extern __shared__ int32_t sm[];
    const int EB = E + 1;                         // buckets: experts, then padding
    int32_t* hist = sm;                           // [kRouteWarps][EB]: rows of bucket e in warp w's block
    int32_t* cnt = hist + kRouteWarps * EB;       // [EB] totals
    uint32_t* sid = reinterpret_cast<uint32_t*>(cnt + EB);  // [M] bucket of each row
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kRouteWarps * EB; i += blockDim.x) hist[i] = 0;
    for (int i = threadIdx.x; i < M; i += blockDim.x) {
        const uint32_t e = ids[i];  // coherent load: ids may be the previous kernel's output
        sid[i] = e < (uint32_t)E ? e : (uint32_t)E;
    }
    __syncthreads();
    const int per = (M + kRouteWarps - 1) / kRouteWarps;
    const int b0 = min(M, warp * per), b1 = min(M, b0 + per);
    for (int i = b0 + lane; i < b1; i += 32) atomicAdd(&hist[warp * EB + sid[i]], 1);
    __syncthreads();
    // totals per bucket, then each warp's running offset inside its bucket
    for (int e = threadIdx.x; e < EB; e += blockDim.x) {
        int run = 0;
        for (int w = 0; w < kRouteWarps; ++w) {
            const int c = hist[w * EB + e];
            hist[w * EB + e] = run;
            run += c;
        }
        cnt[e] = run;
    }
    __syncthreads();
    // exclusive scan over buckets: rows, and items of the real experts
    const int pe = (EB + blockDim.x - 1) / blockDim.x;
    const int e0 = min(EB, (int)threadIdx.x * pe), e1 = min(EB, e0 + pe);
    int rs = 0, ip = 0, z = 0;
    for (int e = e0; e < e1; ++e) {
        rs += cnt[e];
        if (e < E) ip += (cnt[e] + ir - 1) / ir;
    }
    block_exclusive_scan3(rs, ip, z);
    // (block_exclusive_scan3 ends with a barrier: every thread has read cnt)
    const int rs0 = rs;
    {
        int r = rs, p = ip;
        for (int e = e0; e < e1; ++e) {
            const int c = cnt[e];
            if (e < E) {
                row_start[e] = r;
                item_prefix[e] = p;
                for (int q = 0; q < c; q += ir) item_info[p++] = make_int4(e, r + q, min(ir, c - q), 0);
            } else {  // the padding bucket: the totals of the real experts
                row_start[E] = r;
                item_prefix[E] = p;
            }
            r += c;
        }
    }
    __syncthreads();
    // first slot of each bucket: reuse cnt as the bucket start
    {
        int r = rs0;
        for (int e = e0; e < e1; ++e) {
            const int c = cnt[e];
            cnt[e] = r;
            r += c;
        }
    }
    __syncthreads();
    // each warp scatters its block in order
    for (int base = b0; base < b1; base += 32) {
        const int i = base + lane;
        const bool valid = i < b1;
        const uint32_t e = valid ? sid[i] : 0xffffffffu;
        const unsigned same = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(same & ((1u << lane) - 1u));
        int pos = 0;
        if (valid) pos = cnt[e] + hist[warp * EB + e] + rank;
        __syncwarp();
        if (valid && (same >> lane) == 1u) hist[warp * EB + e] += __popc(same);  // the highest lane of each group
        __syncwarp();
        if (valid) {
            order[pos] = (uint32_t)i;
            idx_s[pos] = e;
            row_src[pos] = (uint32_t)i / (uint32_t)top_k;
            inv[i] = (uint32_t)pos;
        }
    }
}

// ---- expert-parallel dispatch: the send buffer of the padded exchange -----------
// Row i = t * top_k + k of a rank's (token, expert) pairs goes to the owner
// d = ids[i] / E_local of its expert, into slot d * cap + (number of earlier
// rows with the same owner): a stable, deterministic packing (the order the
// reference's argsort by owner gives).  A slot is one send row of row_stride
// elements: the token's row x[t] in its first `hidden` elements and the local
// expert id ids[i] - d * E_local as an int32 right after them, so one
// all-to-all carries rows and ids together.  slot_of[i] = s is what the
// combine later reads back.  One CTA per row: one pass over the ids gives its
// place among its owner's rows and every owner's row count (n <= a few
// thousand: a few KB of L2 reads), then it copies its 16-byte chunks.  The
// CTA also writes the padding id E_local into the slots i * world ..
// i * world + world - 1 that no row claims (their x elements are ignored).
constexpr int kEpMaxWorld = 256;
__global__ void ep_pack_kernel(const int32_t* ids, int n, int e_local, int world, int top_k, int cap,
                               const uint16_t* __restrict__ x, int hidden, uint16_t* __restrict__ send,
                               int row_stride, int32_t* slot_of) {
    __shared__ int warp_counts[32];
    __shared__ int owner_counts[kEpMaxWorld];
    const int i = blockIdx.x;
    for (int o = threadIdx.x; o < world; o += blockDim.x) owner_counts[o] = 0;
    __syncthreads();
    const int e = ids[i];
    const int d = e / e_local;
    const bool in_range = e >= 0 && d < world;
    // one pass over the ids: this row's place among its owner's rows, and
    // every owner's row count (for the padding ids below)
    int c = 0;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const int ej = ids[j], dj = ej / e_local;
        if (ej >= 0 && dj < world) {
            atomicAdd(&owner_counts[dj], 1);
            c += (j < i && dj == d) ? 1 : 0;
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) warp_counts[wid] = c;
    __syncthreads();
    int pos = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) pos += warp_counts[w];
    // slots i*world .. i*world + world - 1 that no row claims get the padding
    // id e_local (the slots of owner dd beyond its row count)
    for (int q = threadIdx.x; q < world; q += blockDim.x) {
        const long long s2 = (long long)i * world + q;
        const int dd = (int)(s2 / cap), pp = (int)(s2 - (long long)dd * cap);
        if (pp >= owner_counts[dd]) *reinterpret_cast<int32_t*>(send + s2 * row_stride + hidden) = e_local;
    }
    if (!in_range) {  // an id outside [0, e_local * world): no slot (its combine term reads slot 0)
        if (threadIdx.x == 0) slot_of[i] = 0;
        return;
    }
    const long long slot = (long long)d * cap + pos;
    if (threadIdx.x == 0) {
        *reinterpret_cast<int32_t*>(send + slot * row_stride + hidden) = e - d * e_local;
        slot_of[i] = (int32_t)slot;
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + (long long)(i / top_k) * hidden);
    uint4* dst = reinterpret_cast<uint4*>(send + slot * row_stride);
    for (int q = threadIdx.x; q < hidden / 8; q += blockDim.x) dst[q] = src[q];
}

// ---- combine -----------------------------------------------------------------
// y[t, n] = sum_k w[t*top_k+k] * out_sorted[inv[t*top_k+k], n]; one thread per
// 8 consecutive columns (16-byte loads and stores), fp32 accumulation in k order.
// The indices and weights of up to 8 slots are loaded together, then their
// rows, then summed in slot order: two memory round trips per 8 slots instead
// of two per slot.
template <bool F16>
__global__ void moe_combine_kernel(const uint16_t* out_sorted, const uint32_t* inv, const float* wts,
                                   uint16_t* __restrict__ y, int rows, int top_k,
                                   int N, long long src_rows) {
    using H = Half<F16>;
    // no-ops without the programmatic launch attribute; with it (the combine
    // after this library's own down projection), wait before any global access
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.y;
    const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
    const int n0 = c8 * 8;
    if (n0 >= N) return;
    const bool full = n0 + 8 <= N;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int k0 = 0; k0 < top_k; k0 += 8) {
        const int kn = top_k - k0 < 8 ? top_k - k0 : 8;
        uint32_t src[8];
        float wk[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            src[j] = 0xffffffffu;
            wk[j] = 0.0f;
            if (j < kn) {
                const size_t i = (size_t)t * top_k + k0 + j;
                src[j] = ld_dep(inv + i);
                wk[j] = ld_dep(wts + i);
            }
        }
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            v[j] = make_uint4(0, 0, 0, 0);
            if (j < kn && (long long)src[j] < src_rows && full) v[j] = ld_v4(out_sorted + (size_t)src[j] * N + n0);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (j >= kn || (long long)src[j] >= src_rows) continue;  // out-of-range index: skipped
            if (full) {
                const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    acc[2 * q] = fmaf(wk[j], H::to_f32((uint16_t)(u[q] & 0xffffu)), acc[2 * q]);
                    acc[2 * q + 1] = fmaf(wk[j], H::to_f32((uint16_t)(u[q] >> 16)), acc[2 * q + 1]);
                }
            } else {
                const uint16_t* p = out_sorted + (size_t)src[j] * N + n0;
                for (int q = 0; q < N - n0; ++q) acc[q] = fmaf(wk[j], H::to_f32(p[q]), acc[q]);
            }
        }
    }
    uint16_t* q = y + (size_t)t * N + n0;
    if (full) {
        uint4 o;
        o.x = H::pack2(acc[0], acc[1]);
        o.y = H::pack2(acc[2], acc[3]);
        o.z = H::pack2(acc[4], acc[5]);
        o.w = H::pack2(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(q) = o;
    } else {
        for (int j = 0; j < N - n0; ++j) q[j] = H::from_f32(acc[j]);
    }
}

// ---- dequantise ----------------------------------------------------------------
// out[n, k] = T(s * q + b), the fp32 value rounded once to T (the steel loader's
// static_cast<U>(s*q+b), quantized.h:483-569).
template <bool F16>
__global__ void dequantize_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ sc,
                                  const uint16_t* __restrict__ bi, uint16_t* __restrict__ out, long long N, int K,
                                  int gs, int bits) {
    using H = Half<F16>;
    const long long total = N * (long long)K;
    const long long wrow = (long long)K * bits / 32;
    const int G = K / gs;
    for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long n = idx / K;
        const int k = (int)(idx - n * K);
        const long long bit = (long long)k * bits;
        const uint32_t* row = w + n * wrow;
        const long long word = bit >> 5;
        const int off = (int)(bit & 31);
        unsigned long long v = row[word];
        if (off + bits > 32) v |= (unsigned long long)row[word + 1] << 32;
        const uint32_t q = (uint32_t)(v >> off) & ((1u << bits) - 1u);
        const float s = H::to_f32(sc[n * G + k / gs]);
        const float b = H::to_f32(bi[n * G + k / gs]);
        out[idx] = H::from_f32(__fadd_rn(__fmul_rn(s, (float)q), b));
    }
}

// out[s] = lhs[order[s]]
__global__ void compose_kernel(const int32_t* __restrict__ lhs, const uint32_t* __restrict__ order, uint32_t* out,
                               long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = (uint32_t)lhs[order[i]];
}

}  // namespace qmm

namespace qmm_host {

int launch_compose(const int32_t* lhs, const uint32_t* order, uint32_t* out, long long n, cudaStream_t st) {
    const long long blocks = (n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024;
    qmm::compose_kernel<<<(unsigned)(blocks > 0 ? blocks : 1), 256, 0, st>>>(lhs, order, out, n);
    return cuda_status(cudaGetLastError(), "compose launch");
}

int launch_segment_tables(const int32_t* ids, int M, const int32_t* counts_in, int E, int bm, int mix,
                          int32_t* counts, int32_t* row_start, int32_t* tile_prefix, int32_t* item_prefix,
                          int item_rows, int4* item_info, cudaStream_t st) {
    const size_t smem = (size_t)E * sizeof(int32_t);
    if (smem > 200 * 1024) {
        set_error("segment_tables: E=%d too large", E);
        return QMM_EUNSUPPORTED;
    }
    if (smem > 48 * 1024) {
        const int rc0 = ensure_smem_limit((const void*)qmm::segment_tables_kernel, (int)smem, "segment_tables smem");
        if (rc0) return rc0;
    }
    qmm::segment_tables_kernel<<<1, 1024, smem, st>>>(ids, M, counts_in, E, bm, mix, counts, row_start,
                                                       tile_prefix, item_prefix, item_rows, item_info);
    return cuda_status(cudaGetLastError(), "segment_tables launch");
}

int launch_item_prefix(const int32_t* row_start, int E, int32_t* item_prefix, int item_rows, int4* item_info,
                       cudaStream_t st) {
    qmm::item_prefix_from_row_start_kernel<<<1, 1024, 0, st>>>(row_start, E, item_prefix, item_rows, item_info);
    return cuda_status(cudaGetLastError(), "item_prefix launch");
}

size_t sort_workspace(long long M, long long E) {
    const long long B = (M + qmm::kSortBlock - 1) / qmm::kSortBlock;
    return (size_t)((E + 1) * (B > 0 ? B : 1)) * sizeof(int32_t) + 256;
}

int launch_ep_pack(const int32_t* ids, int n, int e_local, int world, int top_k, int cap, const uint16_t* x,
                   int hidden, uint16_t* send, int row_stride, int32_t* slot_of, cudaStream_t st) {
    if (n == 0) return QMM_OK;
    if (world > qmm::kEpMaxWorld) {
        set_error("ep_pack: world=%d > %d", world, qmm::kEpMaxWorld);
        return QMM_EUNSUPPORTED;
    }
    qmm::ep_pack_kernel<<<n, 256, 0, st>>>(ids, n, e_local, world, top_k, cap, x, hidden, send, row_stride, slot_of);
    return cuda_status(cudaGetLastError(), "ep_pack launch");
}

// Shared memory of the route kernel; 0 when (M, E) is outside it.
size_t route_smem(long long M, long long E) {
    if (M < 1 || M > qmm::kRouteMaxRows || E < 1 || E > qmm::kRouteMaxExperts) return 0;
    return (size_t)(qmm::kRouteWarps + 1) * (size_t)(E + 1) * 4 + (size_t)M * 4;
}

int launch_moe_route(const uint32_t* ids, int M, int E, int top_k, int ir, uint32_t* order, uint32_t* idx_s,
                     uint32_t* row_src, uint32_t* inv, int32_t* row_start, int32_t* item_prefix, int4* item_info,
                     cudaStream_t st) {
    const size_t smem = route_smem(M, E);
    if (!smem) {
        set_error("moe_route: M=%d E=%d outside the one-CTA route (M <= %d, E <= %d)", M, E, qmm::kRouteMaxRows,
                  qmm::kRouteMaxExperts);
        return QMM_EUNSUPPORTED;
    }
    if (smem > 48 * 1024) {
        const int rc = ensure_smem_limit((const void*)qmm::moe_route_kernel, (int)smem, "moe_route smem");
        if (rc) return rc;
    }
    // a plain launch: the ids may come from work this library does not own
    // (a router kernel, or a collective's cross-stream join)
    qmm::moe_route_kernel<<<1, qmm::kRouteThreads, smem, st>>>(ids, M, E, top_k, ir, order, idx_s, row_src, inv,
                                                                row_start, item_prefix, item_info);
    return cuda_status(cudaGetLastError(), "moe_route launch");
}

int launch_sort_rows(const uint32_t* ids, int M, int E, int top_k, uint32_t* order, uint32_t* idx_s,
                     uint32_t* row_src, uint32_t* inv, void* ws, size_t ws_bytes, cudaStream_t st) {
    if (M == 0) return QMM_OK;
    const int B = (M + qmm::kSortBlock - 1) / qmm::kSortBlock;
    if (ws_bytes < sort_workspace(M, E)) {
        set_error("sort_rows: workspace %zu < %zu bytes", ws_bytes, sort_workspace(M, E));
        return QMM_EINVAL;
    }
    const size_t smem = (size_t)(E + 1) * sizeof(int32_t);
    if (smem > 200 * 1024) {
        set_error("sort_rows: E=%d too large", E);
        return QMM_EUNSUPPORTED;
    }
    if (smem > 48 * 1024) {
        int rc0 = ensure_smem_limit((const void*)qmm::sort_hist_kernel, (int)smem, "sort_hist smem");
        if (!rc0) rc0 = ensure_smem_limit((const void*)qmm::sort_scatter_kernel, (int)smem, "sort_scatter smem");
        if (rc0) return rc0;
    }
    int32_t* hist = static_cast<int32_t*>(ws);
    qmm::sort_hist_kernel<<<B, 256, smem, st>>>(ids, M, E, B, hist);
    int rc = cuda_status(cudaGetLastError(), "sort_hist launch");
    if (rc) return rc;
    qmm::exclusive_scan_kernel<<<1, 1024, 0, st>>>(hist, (E + 1) * B);
    rc = cuda_status(cudaGetLastError(), "sort_scan launch");
    if (rc) return rc;
    qmm::sort_scatter_kernel<<<B, 256, smem, st>>>(ids, M, E, B, top_k, hist, order, idx_s, row_src, inv);
    return cuda_status(cudaGetLastError(), "sort_scatter launch");
}

// pdl: launch with programmatic stream serialization (only when the previous
// kernel of the stream is this library's own gathered matmul).
int launch_moe_combine(const uint16_t* out_sorted, long long src_rows, const uint32_t* inv, const float* w,
                       uint16_t* y, int rows, int top_k, int N, bool f16, cudaStream_t st, bool pdl) {
    if (rows == 0 || N == 0) return QMM_OK;
    const int c8 = (N + 7) / 8;
    const int threads = c8 < 128 ? ((c8 + 31) / 32) * 32 : 128;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((c8 + threads - 1) / threads, rows);
    cfg.blockDim = dim3(threads);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
    const cudaError_t e = f16 ? cudaLaunchKernelEx(&cfg, qmm::moe_combine_kernel<true>, out_sorted, inv, w, y, rows,
                                                   top_k, N, src_rows)
                              : cudaLaunchKernelEx(&cfg, qmm::moe_combine_kernel<false>, out_sorted, inv, w, y, rows,
                                                   top_k, N, src_rows);
    if (e != cudaSuccess) cudaGetLastError();
    return cuda_status(e, "moe_combine launch");
}

int launch_dequantize(const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* out, long long N, int K,
                      int gs, int bits, bool f16, cudaStream_t st) {
    const long long total = N * K;
    if (total == 0) return QMM_OK;
    long long blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (f16) qmm::dequantize_kernel<true><<<(unsigned)blocks, 256, 0, st>>>(w, sc, bi, out, N, K, gs, bits);
    else qmm::dequantize_kernel<false><<<(unsigned)blocks, 256, 0, st>>>(w, sc, bi, out, N, K, gs, bits);
    return cuda_status(cudaGetLastError(), "dequantize launch");
}

}  // namespace qmm_host
