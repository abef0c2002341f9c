// capi.cu -- the extern "C" boundary of libmlxturbo_b200.so (include/mlxturbo_b200.h).
//
// Every entry point validates shapes, dtypes and alignment, chooses the
// kernel for the regime and returns a qmm_status.  There is no CPU path and no
// fallback: a request outside what the kernels implement returns
// QMM_EUNSUPPORTED with a message in qmm_last_error().

#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "common.cuh"

#include "qmv_args.cuh"

namespace qmm_host {

// ---- errors -----------------------------------------------------------------
static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int cuda_status(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return QMM_OK;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return QMM_ECUDA;
}

// ---- fire counters (mlxturbo/kernels/_fire.py:1-32) ---------------------------
static const char* const kFireNames[] = {
    "qmv",       "qmv_gather", "qmm_prefill", "segment_tables", "sort_rows", "moe_combine",
    "dequantize", "qmv_chunked", "qmv_i8",     "moe_glu_decode",
};
constexpr int kNumFire = sizeof(kFireNames) / sizeof(kFireNames[0]);
static std::atomic<long long> g_fire[kNumFire];

void fire(const char* name) {
    for (int i = 0; i < kNumFire; ++i)
        if (strcmp(kFireNames[i], name) == 0) {
            g_fire[i].fetch_add(1, std::memory_order_relaxed);
            return;
        }
}

// ---- launchers defined in the other translation units -------------------------
int qmv_k_warps(long long N, long long K, int gs);
int qmv_rows_per_warp(long long N);
bool qmv_cta_preferred(long long N, long long K, int gs, int bits, int* rw, int* kw, int* kc);
bool qmv_cta_preferred_wide(long long N, long long K, int gs, int bits, int* rw, int* kw);
int launch_qmv_stages(const qmm::QmvArgs& a, int mt, int rw, int k_warps, int stages, cudaStream_t st);
template <bool GATHER>
int launch_qmv(const qmm::QmvArgs& a, int bits, int gs, bool f16, int mt, int rw, int k_warps, int grid_y,
               cudaStream_t st);
int launch_segment_tables(const int32_t* ids, int M, const int32_t* counts_in, int E, int bm, int mix,
                          int32_t* counts, int32_t* row_start, int32_t* tile_prefix, int32_t* item_prefix,
                          int item_rows, int4* item_info, cudaStream_t st);
int launch_item_prefix(const int32_t* row_start, int E, int32_t* item_prefix, int item_rows, int4* item_info,
                       cudaStream_t st);
size_t sk_gather_workspace();
int sk_gather_item_rows(long long rows, long long E);
long long sk_gather_items_max(long long rows, long long E);
bool sk_gather_fits(long long rows, long long E, long long N);
int launch_qmv_sk_gather(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                         const int4* item_info, const int32_t* n_items, const uint32_t* row_src,
                         const uint32_t* row_dst, const float* row_scale, long long rows, long long x_rows,
                         long long E, int N, int K, int gs, int bits, bool f16, void* ws, cudaStream_t st, int glu,
                         long long x_stride);
size_t sort_workspace(long long M, long long E);
size_t route_smem(long long M, long long E);
int launch_ep_pack(const int32_t* ids, int n, int e_local, int world, int top_k, int cap, const uint16_t* x,
                   int hidden, uint16_t* send, int row_stride, int32_t* slot_of, cudaStream_t st);
int launch_moe_route(const uint32_t* ids, int M, int E, int top_k, int ir, uint32_t* order, uint32_t* idx_s,
                     uint32_t* row_src, uint32_t* inv, int32_t* row_start, int32_t* item_prefix, int4* item_info,
                     cudaStream_t st);
int launch_sort_rows(const uint32_t* ids, int M, int E, int top_k, uint32_t* order, uint32_t* idx_s,
                     uint32_t* row_src, uint32_t* inv, void* ws, size_t ws_bytes, cudaStream_t st);
int launch_moe_combine(const uint16_t* out_sorted, long long src_rows, const uint32_t* inv, const float* w,
                       uint16_t* y, int rows, int top_k, int N, bool f16, cudaStream_t st, bool pdl);
int launch_dequantize(const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* out, long long N, int K,
                      int gs, int bits, bool f16, cudaStream_t st);
int launch_compose(const int32_t* lhs, const uint32_t* order, uint32_t* out, long long n, cudaStream_t st);
int launch_quantize(const float* w, uint32_t* wq, uint16_t* sc, uint16_t* bi, long long N, int K, int gs, int bits,
                    bool f16, cudaStream_t st);
size_t sk_workspace(long long M, long long N, long long K, int gs, int bits);
bool i8_eligible(long long M, long long N, long long K, int gs, int bits, const void* sc, const void* bi);
bool i8_supported(long long M, long long N, long long K, int gs, int bits, const void* sc, const void* bi);
size_t i8_total_workspace(long long M, long long N, long long K, int gs, int bits);
int launch_qmv_i8(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st,
                  unsigned long long* amax = nullptr, long long n_offset = 0);
int launch_qmv_sk(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st);
int prefill_supported(int bits, int gs);
int launch_prefill(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y,
                   long long M, long long N, long long K, int gs, int bits, bool f16, cudaStream_t st,
                   int force_bt = 0);
int device_error(int reset);
int launch_row_argmax(const uint16_t* y, int M, int N, long long n_offset, unsigned long long* keys, bool f16,
                      cudaStream_t st);

}  // namespace qmm_host

using namespace qmm_host;

namespace qmm_host {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Codes, group size, dtype and (N, K) every matmul entry point accepts.
int check_quant(int64_t N, int64_t K, int group_size, int bits, int dtype) {
    if (dtype != QMM_BF16 && dtype != QMM_F16) {
        set_error("dtype %d: activations must be bf16 or fp16", dtype);
        return QMM_EUNSUPPORTED;
    }
    if (bits != 4 && bits != 8) {
        set_error("bits=%d: kernels implement 4- and 8-bit affine codes", bits);
        return QMM_EUNSUPPORTED;
    }
    if (group_size != 32 && group_size != 64 && group_size != 128) {
        set_error("group_size=%d: must be 32, 64 or 128", group_size);
        return QMM_EUNSUPPORTED;
    }
    if (N <= 0 || K <= 0 || K % group_size != 0) {
        set_error("bad shape N=%lld K=%lld group_size=%d", (long long)N, (long long)K, group_size);
        return QMM_EINVAL;
    }
    if (K > (1LL << 30) || N > (1LL << 30)) {
        set_error("N=%lld K=%lld exceed the 2^30 limit", (long long)N, (long long)K);
        return QMM_EUNSUPPORTED;
    }
    return QMM_OK;
}

// Pointers of a dense matmul: non-null; x, w and y 16-byte aligned, scales
// and biases 2-byte aligned.
int check_dense_pointers(const void* x, const void* w, const void* scales, const void* biases, const void* y) {
    if (!x || !w || !scales || !biases || !y) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || ((uintptr_t)scales & 1u) || ((uintptr_t)biases & 1u)) {
        set_error("x, w and y must be 16-byte aligned, scales and biases 2-byte aligned");
        return QMM_EINVAL;
    }
    return QMM_OK;
}

}  // namespace qmm_host

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

// Dense M <= 16 rows through the decode kernel.
int run_qmv(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int64_t M,
            int64_t N, int64_t K, int gs, int bits, int dtype, int rw, int kw, cudaStream_t st, int kc = 1) {
    qmm::QmvArgs a{};
    a.x = static_cast<const uint16_t*>(x);
    a.w = w;
    a.sc = static_cast<const uint16_t*>(scales);
    a.bi = static_cast<const uint16_t*>(biases);
    a.y = static_cast<uint16_t*>(y);
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    const int mt = M <= 8 ? 1 : 2;
    return launch_qmv<false>(a, bits, gs, dtype == QMM_F16, mt, rw, kw, kc, st);
}

}  // namespace

extern "C" {

const char* qmm_status_string(int status) {
    switch (status) {
        case QMM_OK: return "QMM_OK";
        case QMM_EUNSUPPORTED: return "QMM_EUNSUPPORTED";
        case QMM_EINVAL: return "QMM_EINVAL";
        case QMM_ECUDA: return "QMM_ECUDA";
        case QMM_ENCCL: return "QMM_ENCCL";
        case QMM_ETIMEOUT: return "QMM_ETIMEOUT";
        default: return "QMM_UNKNOWN";
    }
}

const char* qmm_last_error(void) { return g_err; }

int qmm_version(void) { return 100; }

int qmm_qmv_k_warps(int64_t N, int64_t K, int group_size) {
    if (group_size <= 0 || K <= 0 || N <= 0) return 0;
    return qmv_k_warps(N, K, group_size);
}

size_t qmm_quantized_matmul_workspace_size(int64_t M, int64_t N, int64_t K, int group_size, int bits) {
    if (M <= 0 || M > 16 || N <= 0 || K <= 0 || group_size <= 0 || bits <= 0) return 0;
    if (group_size != 32 && group_size != 64 && group_size != 128) return 0;
    const size_t sk = sk_workspace(M, N, K, group_size, bits);
    const size_t i8 = M <= 8 ? i8_total_workspace(M, N, K, group_size, bits) : 0;
    return sk > i8 ? sk : i8;
}

int qmm_quantized_matmul(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                         int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype, void* workspace,
                         size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (M < 0) {
        set_error("M=%lld < 0", (long long)M);
        return QMM_EINVAL;
    }
    if (M == 0) return QMM_OK;
    rc = check_dense_pointers(x, w, scales, biases, y);
    if (rc) return rc;
    cudaStream_t st = as_stream(stream);
    if (M <= 16) {
        fire("qmv");
        if (workspace) {
            if (!aligned16(workspace)) {
                set_error("workspace must be 16-byte aligned");
                return QMM_EINVAL;
            }
            if (i8_eligible(M, N, K, group_size, bits, scales, biases) &&
                workspace_bytes >= i8_total_workspace(M, N, K, group_size, bits)) {
                fire("qmv_i8");
                return launch_qmv_i8(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                                     static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N,
                                     (int)K, group_size, bits, dtype == QMM_F16, workspace, workspace_bytes, st);
            }
            int rw = 0, kw = 0, kc = 1;
            if (qmv_cta_preferred(N, K, group_size, bits, &rw, &kw, &kc) ||
                (M > 8 && qmv_cta_preferred_wide(N, K, group_size, bits, &rw, &kw)))
                return run_qmv(x, w, scales, biases, y, M, N, K, group_size, bits, dtype, rw, kw, st, kc);
            return launch_qmv_sk(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                                 static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N,
                                 (int)K, group_size, bits, dtype == QMM_F16, workspace, workspace_bytes, st);
        }
        return run_qmv(x, w, scales, biases, y, M, N, K, group_size, bits, dtype, qmv_rows_per_warp(N),
                       qmv_k_warps(N, K, group_size), st);
    }
    if (prefill_supported(bits, group_size)) {
        fire("qmm_prefill");
        return launch_prefill(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                              static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), M, N, K, group_size,
                              bits, dtype == QMM_F16, st);
    }
    // Prefill shapes the tensor-core kernel does not cover run as 16-row chunks
    // of the decode kernel (each chunk re-streams the weights).
    fire("qmv_chunked");
    const int kw = qmv_k_warps(N, K, group_size), rw = qmv_rows_per_warp(N);
    for (int64_t m0 = 0; m0 < M; m0 += 16) {
        const int64_t mc = M - m0 < 16 ? M - m0 : 16;
        rc = run_qmv(static_cast<const uint16_t*>(x) + m0 * K, w, scales, biases, static_cast<uint16_t*>(y) + m0 * N,
                     mc, N, K, group_size, bits, dtype, rw, kw, st);
        if (rc) return rc;
    }
    return QMM_OK;
}

int qmm_quantized_matmul_argmax(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y,
                                int64_t M, int64_t N, int64_t K, int group_size, int bits, int dtype,
                                int64_t index_offset, uint64_t* keys, void* workspace, size_t workspace_bytes,
                                void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (M < 0 || M > 65535 || index_offset < 0 || index_offset + N > 0xFFFFFFFFLL) {
        set_error("argmax: M=%lld index_offset=%lld N=%lld out of range", (long long)M, (long long)index_offset,
                  (long long)N);
        return QMM_EINVAL;
    }
    if (M == 0) return QMM_OK;
    rc = check_dense_pointers(x, w, scales, biases, y);
    if (rc) return rc;
    if (!keys || ((uintptr_t)keys & 7u)) {
        set_error("argmax: keys must be an 8-byte aligned device array of M words");
        return QMM_EINVAL;
    }
    cudaStream_t st = as_stream(stream);
    rc = cuda_status(cudaMemsetAsync(keys, 0, (size_t)M * 8, st), "argmax: clearing the keys");
    if (rc) return rc;
    unsigned long long* k = reinterpret_cast<unsigned long long*>(keys);
    if (M <= 16 && workspace && aligned16(workspace) && i8_eligible(M, N, K, group_size, bits, scales, biases) &&
        workspace_bytes >= i8_total_workspace(M, N, K, group_size, bits)) {
        fire("qmv");
        fire("qmv_i8");
        return launch_qmv_i8(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                             static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N, (int)K,
                             group_size, bits, dtype == QMM_F16, workspace, workspace_bytes, st, k, index_offset);
    }
    rc = qmm_quantized_matmul(x, w, scales, biases, y, M, N, K, group_size, bits, dtype, workspace, workspace_bytes,
                              stream);
    if (rc) return rc;
    return launch_row_argmax(static_cast<const uint16_t*>(y), (int)M, (int)N, index_offset, k, dtype == QMM_F16, st);
}

int qmm_qmv_i8(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int64_t M,
               int64_t N, int64_t K, int group_size, int bits, int dtype, void* workspace, size_t workspace_bytes,
               void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (!x || !w || !scales || !biases || !y || !workspace) {
        set_error("qmv_i8: null pointer argument");
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || !aligned16(workspace)) {
        set_error("qmv_i8: x, w, y and workspace must be 16-byte aligned");
        return QMM_EINVAL;
    }
    if (!i8_supported(M, N, K, group_size, bits, scales, biases)) {
        set_error("qmv_i8: M=%lld N=%lld K=%lld group_size=%d bits=%d outside the kernel's shapes", (long long)M,
                  (long long)N, (long long)K, group_size, bits);
        return QMM_EUNSUPPORTED;
    }
    fire("qmv_i8");
    return launch_qmv_i8(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                         static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N, (int)K,
                         group_size, bits, dtype == QMM_F16, workspace, workspace_bytes, as_stream(stream));
}

int qmm_qmv_explicit(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int64_t M,
                     int64_t N, int64_t K, int group_size, int bits, int dtype, int rows_per_warp, int k_warps,
                     void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    const int rw_ = rows_per_warp % 10;
    if (M < 1 || M > 16 || (rw_ != 1 && rw_ != 2) || k_warps < 1 || k_warps > 16) {
        set_error("qmv_explicit: M=%lld rows_per_warp=%d k_warps=%d out of range", (long long)M, rows_per_warp,
                  k_warps);
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y)) {
        set_error("x, w and y must be 16-byte aligned");
        return QMM_EINVAL;
    }
    fire("qmv");
    if (rows_per_warp >= 10) {  // tuning: rows_per_warp = 10*stages + rw (4-bit g64 bf16 only)
        qmm::QmvArgs a{};
        a.x = static_cast<const uint16_t*>(x);
        a.w = w;
        a.sc = static_cast<const uint16_t*>(scales);
        a.bi = static_cast<const uint16_t*>(biases);
        a.y = static_cast<uint16_t*>(y);
        a.M = (int)M;
        a.N = (int)N;
        a.K = (int)K;
        return launch_qmv_stages(a, M <= 8 ? 1 : 2, rows_per_warp % 10, k_warps, rows_per_warp / 10, as_stream(stream));
    }
    return run_qmv(x, w, scales, biases, y, M, N, K, group_size, bits, dtype, rows_per_warp, k_warps,
                   as_stream(stream));
}

// Gather / segmented workspace, in this order (each part 256-byte aligned):
//   [stream-K block]  tile counters (zero between calls) + partial-sum slots
//   row_start, item_prefix (E+1 each), item_info (int4 per item)
//   gather only: order, idx_s, row_src, inv (rows each), sort scratch
static size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }

struct GatherWs {
    char* sk;
    int32_t* row_start;
    int32_t* item_prefix;
    int4* item_info;
    char* rest;
};

static GatherWs gather_ws(void* base, int64_t rows, int64_t E) {
    GatherWs g;
    char* p = static_cast<char*>(base);
    g.sk = p;
    p += al256(sk_gather_workspace());
    g.row_start = reinterpret_cast<int32_t*>(p);
    g.item_prefix = g.row_start + (E + 1);
    p += al256((size_t)(2 * (E + 1)) * 4);
    g.item_info = reinterpret_cast<int4*>(p);
    p += al256((size_t)sk_gather_items_max(rows, E) * sizeof(int4));
    g.rest = p;
    return g;
}

size_t qmm_segmented_workspace_size(int64_t M, int64_t E) {
    return al256(sk_gather_workspace()) + al256((size_t)(2 * (E + 1)) * 4) +
           al256((size_t)sk_gather_items_max(M, E) * sizeof(int4));
}

size_t qmm_gather_workspace_size(int64_t rows, int64_t E) {
    return qmm_segmented_workspace_size(rows, E) + al256((size_t)(4 * rows) * 4) + sort_workspace(rows, E);
}

// Sorted rows with the expert segments in `row_start`: the stream-K gather
// kernel when its tile counters cover the problem, else the CTA-per-item
// kernel (qmv.cu, 16-row items).  Builds the item tables itself when the
// caller passes only row_start (tables_ready = false).
static int run_segments(const void* x, const uint32_t* w, const void* scales, const void* biases,
                        const GatherWs& g, const uint32_t* row_src, const uint32_t* row_dst, const float* row_scale,
                        void* y, int64_t M, int64_t x_rows, int64_t E, int64_t N, int64_t K, int gs, int bits,
                        int dtype, cudaStream_t st) {
    const bool sk = sk_gather_fits(M, E, N);
    const int ir = sk ? sk_gather_item_rows(M, E) : 16;
    int rc = launch_item_prefix(g.row_start, (int)E, g.item_prefix, ir, sk ? g.item_info : nullptr, st);
    if (rc) return rc;
    if (sk) {
        fire("qmv_gather");
        return launch_qmv_sk_gather(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                                    static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), g.item_info,
                                    g.item_prefix + E, row_src, row_dst, row_scale, M, x_rows, E, (int)N, (int)K, gs,
                                    bits, dtype == QMM_F16, g.sk, st, 0, 0);
    }
    qmm::QmvArgs a{};
    a.x = static_cast<const uint16_t*>(x);
    a.w = w;
    a.sc = static_cast<const uint16_t*>(scales);
    a.bi = static_cast<const uint16_t*>(biases);
    a.y = static_cast<uint16_t*>(y);
    a.M = 16;
    a.N = (int)N;
    a.K = (int)K;
    a.seg.row_start = g.row_start;
    a.seg.tile_prefix = g.item_prefix;
    a.seg.row_src = row_src;
    a.seg.row_dst = row_dst;
    a.seg.row_scale = row_scale;
    a.seg.E = (int)E;
    a.seg.x_rows = (int)x_rows;
    a.seg.y_rows = (int)M;
    a.seg.w_stride = N * (K * bits / 32);
    a.seg.s_stride = N * (K / gs);
    const long long items_max = (M + 15) / 16 + (E < M ? E : M);
    if (items_max > 65535) {
        set_error("gather: %lld rows need %lld row items (limit 65535)", (long long)M, items_max);
        return QMM_EUNSUPPORTED;
    }
    const int mt = M <= 8 ? 1 : 2;
    fire("qmv_gather");
    return launch_qmv<true>(a, bits, gs, dtype == QMM_F16, mt, qmv_rows_per_warp(N), qmv_k_warps(N, K, gs),
                            (int)items_max, st);
}

int qmm_gather_qmm(const void* x, const uint32_t* w, const void* scales, const void* biases,
                   const int32_t* lhs_indices, const int32_t* rhs_indices, void* y, int64_t rows, int64_t x_rows,
                   int64_t E, int64_t N, int64_t K, int group_size, int bits, int dtype, int sorted_indices,
                   void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (rows < 0 || E <= 0 || x_rows < 0) {
        set_error("bad gather shape rows=%lld E=%lld", (long long)rows, (long long)E);
        return QMM_EINVAL;
    }
    if (rows == 0) return QMM_OK;
    if (!x || !w || !scales || !biases || !y || !rhs_indices || !workspace) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || !aligned16(workspace)) {
        set_error("x, w, y and workspace must be 16-byte aligned");
        return QMM_EINVAL;
    }
    if (workspace_bytes < qmm_gather_workspace_size(rows, E)) {
        set_error("gather workspace %zu < %zu bytes", workspace_bytes, qmm_gather_workspace_size(rows, E));
        return QMM_EINVAL;
    }
    if (rows > (1LL << 30) || E > 16384) {
        set_error("rows=%lld E=%lld beyond limits", (long long)rows, (long long)E);
        return QMM_EUNSUPPORTED;
    }
    cudaStream_t st = as_stream(stream);
    const GatherWs g = gather_ws(workspace, rows, E);
    uint32_t* order = reinterpret_cast<uint32_t*>(g.rest);
    uint32_t* idx_s = order + rows;
    uint32_t* row_src = idx_s + rows;
    uint32_t* inv = row_src + rows;
    char* sort_ws = g.rest + al256((size_t)(4 * rows) * 4);
    const size_t sort_bytes = workspace_bytes - (size_t)(sort_ws - static_cast<char*>(workspace));

    if (sorted_indices) {
        fire("segment_tables");
        rc = launch_segment_tables(rhs_indices, (int)rows, nullptr, (int)E, 16, 0, nullptr, g.row_start, nullptr,
                                   nullptr, 16, nullptr, st);
        if (rc) return rc;
        return run_segments(x, w, scales, biases, g, reinterpret_cast<const uint32_t*>(lhs_indices), nullptr, nullptr,
                            y, rows, x_rows, E, N, K, group_size, bits, dtype, st);
    }
    // Unsorted: sort rows by expert on the device, gather x rows through the
    // permutation and scatter outputs back to the caller's row order.
    fire("sort_rows");
    rc = launch_sort_rows(reinterpret_cast<const uint32_t*>(rhs_indices), (int)rows, (int)E, 1, order, idx_s, row_src,
                          inv, sort_ws, sort_bytes, st);
    if (rc) return rc;
    fire("segment_tables");
    rc = launch_segment_tables(reinterpret_cast<const int32_t*>(idx_s), (int)rows, nullptr, (int)E, 16, 0, nullptr,
                               g.row_start, nullptr, nullptr, 16, nullptr, st);
    if (rc) return rc;
    // x row of sorted row s is lhs[order[s]] (or order[s]); output row is order[s].
    const uint32_t* src = order;
    if (lhs_indices) {
        // compose on the device: row_src[s] = lhs[order[s]]
        rc = launch_compose(lhs_indices, order, row_src, rows, st);
        if (rc) return rc;
        src = row_src;
    }
    return run_segments(x, w, scales, biases, g, src, order, nullptr, y, rows, x_rows, E, N, K, group_size, bits,
                        dtype, st);
}

int qmm_segmented(const void* x, const uint32_t* w, const void* scales, const void* biases, const int32_t* row_start,
                  const uint32_t* row_src, const uint32_t* row_dst, const float* row_scale, void* y, int64_t M,
                  int64_t x_rows, int64_t E, int64_t N, int64_t K, int group_size, int bits, int dtype,
                  void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (M < 0 || E <= 0 || (row_src && x_rows <= 0)) {
        set_error("bad segmented shape M=%lld E=%lld", (long long)M, (long long)E);
        return QMM_EINVAL;
    }
    if (M == 0) return QMM_OK;
    if (!x || !w || !scales || !biases || !y || !row_start || !workspace) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y)) {
        set_error("x, w and y must be 16-byte aligned");
        return QMM_EINVAL;
    }
    if (workspace_bytes < qmm_segmented_workspace_size(M, E)) {
        set_error("segmented workspace %zu < %zu bytes", workspace_bytes, qmm_segmented_workspace_size(M, E));
        return QMM_EINVAL;
    }
    cudaStream_t st = as_stream(stream);
    GatherWs g = gather_ws(workspace, M, E);
    // the caller's segment starts: copy them beside the item tables
    const cudaError_t e = cudaMemcpyAsync(g.row_start, row_start, (size_t)(E + 1) * 4, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e, "segmented: row_start copy");
    return run_segments(x, w, scales, biases, g, row_src, row_dst, row_scale, y, M, row_src ? x_rows : M, E, N, K,
                        group_size, bits, dtype, st);
}

int qmm_gather_tables(const int32_t* ids_sorted, int64_t rows, int64_t E, void* workspace, size_t workspace_bytes,
                      void* stream) {
    g_err[0] = 0;
    if (rows <= 0 || E <= 0 || E > 16384 || rows > (1LL << 30) || !ids_sorted || !workspace) {
        set_error("gather_tables: bad arguments rows=%lld E=%lld", (long long)rows, (long long)E);
        return QMM_EINVAL;
    }
    if (workspace_bytes < qmm_segmented_workspace_size(rows, E)) {
        set_error("gather_tables: workspace %zu < %zu bytes", workspace_bytes, qmm_segmented_workspace_size(rows, E));
        return QMM_EINVAL;
    }
    const GatherWs g = gather_ws(workspace, rows, E);
    fire("segment_tables");
    return launch_segment_tables(ids_sorted, (int)rows, nullptr, (int)E, 16, 0, nullptr, g.row_start, nullptr,
                                 g.item_prefix, sk_gather_item_rows(rows, E), g.item_info, as_stream(stream));
}

int qmm_moe_route(const int32_t* ids, int64_t rows, int64_t E, int top_k, uint32_t* order, uint32_t* idx_s,
                  uint32_t* row_src, uint32_t* inv, void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (rows <= 0 || E <= 0 || top_k <= 0 || !ids || !order || !idx_s || !row_src || !inv || !workspace) {
        set_error("moe_route: bad arguments rows=%lld E=%lld top_k=%d", (long long)rows, (long long)E, top_k);
        return QMM_EINVAL;
    }
    if (!route_smem(rows, E)) {
        set_error("moe_route: rows=%lld E=%lld outside the one-launch route; use qmm_sort_rows + qmm_gather_tables",
                  (long long)rows, (long long)E);
        return QMM_EUNSUPPORTED;
    }
    if (!aligned16(workspace) || workspace_bytes < qmm_segmented_workspace_size(rows, E)) {
        set_error("moe_route: workspace must be 16-byte aligned and hold %zu bytes",
                  qmm_segmented_workspace_size(rows, E));
        return QMM_EINVAL;
    }
    const GatherWs g = gather_ws(workspace, rows, E);
    fire("sort_rows");
    fire("segment_tables");
    return launch_moe_route(reinterpret_cast<const uint32_t*>(ids), (int)rows, (int)E, top_k,
                            sk_gather_item_rows(rows, E), order, idx_s, row_src, inv, g.row_start, g.item_prefix,
                            g.item_info, as_stream(stream));
}

int qmm_ep_pack(const int32_t* ids, int64_t n, int64_t e_local, int64_t world, int top_k, const void* x,
                int64_t hidden, void* send, int64_t row_stride, int32_t* slot_of, void* stream) {
    g_err[0] = 0;
    // every CTA scans all n ids (an O(n^2) pass sized for decode batches)
    if (n < 0 || e_local <= 0 || world <= 0 || top_k <= 0 || hidden <= 0 || n > (1LL << 16) ||
        e_local * world > (1LL << 30)) {
        set_error("ep_pack: bad arguments n=%lld (<= 65536) e_local=%lld world=%lld", (long long)n,
                  (long long)e_local, (long long)world);
        return QMM_EINVAL;
    }
    if (n == 0) return QMM_OK;
    if (!ids || !x || !send || !slot_of || hidden % 8 || row_stride < hidden + 8 || row_stride % 8 ||
        !aligned16(x) || !aligned16(send) || n * world * row_stride > (1LL << 31)) {
        set_error("ep_pack: null pointer, hidden or row_stride not a multiple of 8, row_stride < hidden + 8, "
                  "x / send not 16-byte aligned, or a send buffer past 2^31 elements");
        return QMM_EINVAL;
    }
    return launch_ep_pack(ids, (int)n, (int)e_local, (int)world, top_k, (int)n, static_cast<const uint16_t*>(x),
                          (int)hidden, static_cast<uint16_t*>(send), (int)row_stride, slot_of, as_stream(stream));
}

int qmm_gather_run(const void* x, const uint32_t* w, const void* scales, const void* biases, const uint32_t* row_src,
                   const uint32_t* row_dst, const float* row_scale, void* y, int64_t rows, int64_t x_rows,
                   int64_t x_stride, int64_t E, int64_t N, int64_t K, int group_size, int bits, int dtype, int glu,
                   void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (rows <= 0 || E <= 0 || x_rows <= 0 || (glu && N % 16)) {
        set_error("gather_run: bad shape rows=%lld E=%lld N=%lld glu=%d", (long long)rows, (long long)E, (long long)N,
                  glu);
        return QMM_EINVAL;
    }
    if (!x || !w || !scales || !biases || !y || !workspace) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y) || !aligned16(workspace)) {
        set_error("x, w, y and workspace must be 16-byte aligned");
        return QMM_EINVAL;
    }
    if (x_stride != 0 && (x_stride < K || x_stride % 8)) {
        set_error("gather_run: x_stride=%lld must be 0 or a multiple of 8 that is >= K=%lld", (long long)x_stride,
                  (long long)K);
        return QMM_EINVAL;
    }
    if (workspace_bytes < qmm_segmented_workspace_size(rows, E)) {
        set_error("gather_run: workspace %zu < %zu bytes", workspace_bytes, qmm_segmented_workspace_size(rows, E));
        return QMM_EINVAL;
    }
    if (!sk_gather_fits(rows, E, N)) {
        set_error("gather_run: %lld rows x %lld experts x %lld outputs exceed the tile counters", (long long)rows,
                  (long long)E, (long long)N);
        return QMM_EUNSUPPORTED;
    }
    const GatherWs g = gather_ws(workspace, rows, E);
    fire(glu ? "qmv_gather_glu" : "qmv_gather");
    return launch_qmv_sk_gather(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                                static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), g.item_info,
                                g.item_prefix + E, row_src, row_dst, row_scale, rows, x_rows, E, (int)N, (int)K,
                                group_size, bits, dtype == QMM_F16, g.sk, as_stream(stream), glu ? 1 : 0, x_stride);
}

int qmm_segment_tables(const int32_t* ids, int64_t M, int64_t E, int bm, int mix_threshold, int32_t* counts,
                       int32_t* row_start, int32_t* tile_prefix, void* stream) {
    g_err[0] = 0;
    if (M < 0 || E <= 0 || bm <= 0 || (M > 0 && !ids)) {
        set_error("segment_tables: bad arguments M=%lld E=%lld bm=%d", (long long)M, (long long)E, bm);
        return QMM_EINVAL;
    }
    fire("segment_tables");
    return launch_segment_tables(ids, (int)M, nullptr, (int)E, bm, mix_threshold, counts, row_start, tile_prefix,
                                 nullptr, 16, nullptr, as_stream(stream));
}

int qmm_segment_tables_from_counts(const int32_t* counts, int64_t E, int bm, int mix_threshold, int32_t* row_start,
                                   int32_t* tile_prefix, void* stream) {
    g_err[0] = 0;
    if (E <= 0 || bm <= 0 || !counts) {
        set_error("segment_tables_from_counts: bad arguments E=%lld bm=%d", (long long)E, bm);
        return QMM_EINVAL;
    }
    fire("segment_tables");
    return launch_segment_tables(nullptr, 0, counts, (int)E, bm, mix_threshold, nullptr, row_start, tile_prefix,
                                 nullptr, 16, nullptr, as_stream(stream));
}

size_t qmm_sort_workspace_size(int64_t M, int64_t E) { return sort_workspace(M, E); }

int qmm_sort_rows(const uint32_t* ids, int64_t M, int64_t E, int top_k, uint32_t* order, uint32_t* idx_s,
                  uint32_t* row_src, uint32_t* inv, void* workspace, size_t workspace_bytes, void* stream) {
    g_err[0] = 0;
    if (M < 0 || E <= 0 || top_k <= 0) {
        set_error("sort_rows: bad arguments");
        return QMM_EINVAL;
    }
    if (M > 0 && (!ids || !order || !idx_s || !row_src || !inv || !workspace)) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    fire("sort_rows");
    return launch_sort_rows(ids, (int)M, (int)E, top_k, order, idx_s, row_src, inv, workspace, workspace_bytes,
                            as_stream(stream));
}

static int combine_rows(const void* out_src, int64_t src_rows, const uint32_t* inv, const float* weights, void* y,
                        int64_t rows, int top_k, int64_t N, int dtype, void* stream, bool pdl) {
    g_err[0] = 0;
    if (dtype != QMM_BF16 && dtype != QMM_F16) {
        set_error("dtype %d unsupported", dtype);
        return QMM_EUNSUPPORTED;
    }
    if (rows < 0 || top_k <= 0 || N < 0 || src_rows < 0) {
        set_error("moe_combine: bad arguments");
        return QMM_EINVAL;
    }
    if (rows > 0 && N > 0 && (!out_src || !inv || !weights || !y)) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    if ((N % 8 == 0) && (!aligned16(out_src) || !aligned16(y))) {
        set_error("out_sorted and y must be 16-byte aligned");
        return QMM_EINVAL;
    }
    fire("moe_combine");
    return launch_moe_combine(static_cast<const uint16_t*>(out_src), src_rows, inv, weights, static_cast<uint16_t*>(y),
                              (int)rows, top_k, (int)N, dtype == QMM_F16, as_stream(stream), pdl);
}

int qmm_moe_combine_rows(const void* out_src, int64_t src_rows, const uint32_t* inv, const float* weights, void* y,
                         int64_t rows, int top_k, int64_t N, int dtype, void* stream) {
    return combine_rows(out_src, src_rows, inv, weights, y, rows, top_k, N, dtype, stream, false);
}

int qmm_moe_combine_chained(const void* out_src, int64_t src_rows, const uint32_t* inv, const float* weights, void* y,
                            int64_t rows, int top_k, int64_t N, int dtype, void* stream) {
    return combine_rows(out_src, src_rows, inv, weights, y, rows, top_k, N, dtype, stream, true);
}

size_t qmm_moe_glu_decode_workspace_size(int64_t T, int64_t top_k, int64_t inter) {
    if (T <= 0 || top_k <= 0 || inter <= 0) return 0;
    return moe_decode_workspace(T, top_k, inter);
}

int qmm_moe_glu_decode(const void* x, const int32_t* ids, const float* weights, const uint32_t* gate_up_w,
                       const void* gate_up_scales, const void* gate_up_biases, const uint32_t* down_w,
                       const void* down_scales, const void* down_biases, void* y, int64_t T, int64_t top_k,
                       int64_t E, int64_t hidden, int64_t inter, int group_size, int bits, int dtype,
                       void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (T <= 0 || top_k <= 0 || E <= 0 || hidden <= 0 || inter <= 0 || T > (1 << 20) || top_k > 1024 ||
        E > (1 << 20)) {
        set_error("moe_glu_decode: bad arguments T=%lld top_k=%lld E=%lld hidden=%lld inter=%lld", (long long)T,
                  (long long)top_k, (long long)E, (long long)hidden, (long long)inter);
        return QMM_EINVAL;
    }
    int rc = check_quant(2 * inter, hidden, group_size, bits, dtype);
    if (rc) return rc;
    if ((rc = check_quant(hidden, inter, group_size, bits, dtype))) return rc;
    if ((rc = moe_decode_supported(T, top_k, E, hidden, inter, group_size, bits))) return rc;
    if (!x || !ids || !weights || !y || !gate_up_w || !gate_up_scales || !gate_up_biases || !down_w ||
        !down_scales || !down_biases || !aligned16(x) || !aligned16(y) || !aligned16(gate_up_w) ||
        !aligned16(gate_up_scales) || !aligned16(gate_up_biases) || !aligned16(down_w) || !aligned16(down_scales) ||
        !aligned16(down_biases)) {
        set_error("moe_glu_decode: null pointer, or x, y or a bank not 16-byte aligned");
        return QMM_EINVAL;
    }
    if (!aligned16(workspace) || workspace_bytes < moe_decode_workspace(T, top_k, inter)) {
        set_error("moe_glu_decode: workspace must be 16-byte aligned and hold %zu bytes",
                  moe_decode_workspace(T, top_k, inter));
        return QMM_EINVAL;
    }
    MoeDecodeCall c{};
    c.x = x;
    c.ids = ids;
    c.wts = weights;
    c.guw = gate_up_w;
    c.gus = gate_up_scales;
    c.gub = gate_up_biases;
    c.dnw = down_w;
    c.dns = down_scales;
    c.dnb = down_biases;
    c.y = y;
    c.T = (int)T;
    c.top_k = (int)top_k;
    c.E = (int)E;
    c.H = (int)hidden;
    c.I = (int)inter;
    c.gs = group_size;
    c.bits = bits;
    c.dtype = dtype;
    c.ws = workspace;
    c.st = as_stream(stream);
    fire("moe_glu_decode");
    return launch_moe_glu_decode(c);
}

int qmm_moe_combine(const void* out_sorted, const uint32_t* inv, const float* weights, void* y, int64_t rows,
                    int top_k, int64_t N, int dtype, void* stream) {
    return qmm_moe_combine_rows(out_sorted, rows * top_k, inv, weights, y, rows, top_k, N, dtype, stream);
}

int qmm_dequantize(const uint32_t* w, const void* scales, const void* biases, void* out, int64_t N, int64_t K,
                   int group_size, int bits, int dtype, void* stream) {
    g_err[0] = 0;
    if (dtype != QMM_BF16 && dtype != QMM_F16) {
        set_error("dtype %d unsupported", dtype);
        return QMM_EUNSUPPORTED;
    }
    if (!(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8) ||
        !(group_size == 32 || group_size == 64 || group_size == 128) || K % group_size || (K * bits) % 32 || N < 0) {
        set_error("dequantize: bits=%d group_size=%d K=%lld unsupported", bits, group_size, (long long)K);
        return QMM_EUNSUPPORTED;
    }
    fire("dequantize");
    return launch_dequantize(w, static_cast<const uint16_t*>(scales), static_cast<const uint16_t*>(biases),
                             static_cast<uint16_t*>(out), N, (int)K, group_size, bits, dtype == QMM_F16,
                             as_stream(stream));
}

int qmm_quantize(const float* w, uint32_t* wq, void* scales, void* biases, int64_t N, int64_t K, int group_size,
                 int bits, int dtype, void* stream) {
    g_err[0] = 0;
    if (dtype != QMM_BF16 && dtype != QMM_F16) {
        set_error("dtype %d unsupported", dtype);
        return QMM_EUNSUPPORTED;
    }
    if (!(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8) ||
        !(group_size == 32 || group_size == 64 || group_size == 128) || K <= 0 || K % group_size || N < 0) {
        set_error("quantize: bits=%d group_size=%d K=%lld unsupported", bits, group_size, (long long)K);
        return QMM_EUNSUPPORTED;
    }
    if (N > 0 && (!w || !wq || !scales || !biases)) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    return launch_quantize(w, wq, static_cast<uint16_t*>(scales), static_cast<uint16_t*>(biases), N, (int)K,
                           group_size, bits, dtype == QMM_F16, as_stream(stream));
}

int qmm_prefill_explicit(const void* x, const uint32_t* w, const void* scales, const void* biases, void* y, int64_t M,
                         int64_t N, int64_t K, int group_size, int bits, int dtype, int tokens_per_cta, void* stream) {
    g_err[0] = 0;
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (M < 1 || (tokens_per_cta != 128 && tokens_per_cta != 256)) {
        set_error("prefill_explicit: M=%lld tokens_per_cta=%d", (long long)M, tokens_per_cta);
        return QMM_EINVAL;
    }
    if (!aligned16(x) || !aligned16(w) || !aligned16(y)) {
        set_error("x, w and y must be 16-byte aligned");
        return QMM_EINVAL;
    }
    fire("qmm_prefill");
    return launch_prefill(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                          static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), M, N, K, group_size, bits,
                          dtype == QMM_F16, as_stream(stream), tokens_per_cta);
}

int qmm_device_error(int reset) { return device_error(reset); }

long long qmm_fire_count(const char* name) {
    for (int i = 0; i < kNumFire; ++i)
        if (strcmp(kFireNames[i], name) == 0) return g_fire[i].load();
    return -1;
}

const char* qmm_fire_names(void) {
    static char buf[512];
    if (!buf[0]) {
        for (int i = 0; i < kNumFire; ++i) {
            if (i) strncat(buf, ",", sizeof(buf) - strlen(buf) - 1);
            strncat(buf, kFireNames[i], sizeof(buf) - strlen(buf) - 1);
        }
    }
    return buf;
}

void qmm_fire_reset(void) {
    for (int i = 0; i < kNumFire; ++i) g_fire[i].store(0);
}

}  // extern "C"
