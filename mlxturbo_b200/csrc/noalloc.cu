// noalloc.cu -- the decode matmul (M <= 16) for callers that cannot allocate
// device memory: its scratch lives in a fixed array inside this library.
//
// Who needs it: callers that plan every device byte up front and never call
// cudaMalloc once inference runs -- embedded and edge runtimes with a fixed
// arena, C/FFI hosts that have no allocator binding at all, and serving
// loops whose latency budget forbids an allocation on the first call of a new
// shape.  qmm_quantized_matmul asks them for a workspace; this entry point
// does not.
//
// The scratch is one file-scope __device__ array of kScratchBytes.  Every GPU
// that loads the library holds it until the process exits.  Host code cannot
// use the array's name as a device address (in host code it names a host-side
// stand-in), so the first call on each device, with that device current, asks
// the runtime for the array's device address with cudaGetSymbolAddress and
// remembers it.  That first call also clears the array; it should come before
// any stream capture on that device.
//
// All calls on a device share the array and it keeps the last call's
// contents.  The decode kernel's tile counters must be zero when a call
// starts: each call clears the counters it will use on its stream before the
// kernel runs (the kernel leaves them zero again).  Two calls that overlap on
// the GPU -- different streams, or different host threads without ordering --
// race on the array and give wrong results.

#include <mutex>

#include "common.cuh"
#include "qmv_args.cuh"

namespace {

// The stream-K kernel needs at most 256 KiB of counters + 2 KiB of partial-sum
// slots per warp (at most 2960 warps): about 6 MiB.  The integer-MMA kernel
// keeps its own slots and activation planes after the first 8 MiB: under
// 13 MiB in all for K up to 65536.
constexpr size_t kScratchBytes = 16u << 20;  // 16 MiB per device
constexpr size_t kCounterBytes = 256u << 10;  // the decode kernel's tile counters come first
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set up on first use).
int scratch_for_current_device(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return qmm_host::cuda_status(e, "noalloc: cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) {
        qmm_host::set_error("noalloc: device %d beyond the %d supported", dev, kMaxDevices);
        return QMM_EUNSUPPORTED;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return qmm_host::cuda_status(e, "noalloc: cudaGetSymbolAddress");
        e = cudaMemset(p, 0, kScratchBytes);
        if (e != cudaSuccess) return qmm_host::cuda_status(e, "noalloc: clearing the scratch array");
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return QMM_OK;
}

}  // namespace

namespace qmm_host {
bool qmv_cta_preferred(long long N, long long K, int gs, int bits, int* rw, int* kw, int* kc);
bool qmv_cta_preferred_wide(long long N, long long K, int gs, int bits, int* rw, int* kw);
template <bool GATHER>
int launch_qmv(const qmm::QmvArgs& a, int bits, int gs, bool f16, int mt, int rw, int k_warps, int grid_y,
               cudaStream_t st);
size_t sk_workspace(long long M, long long N, long long K, int gs, int bits);
int launch_qmv_sk(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st);
bool i8_eligible(long long M, long long N, long long K, int gs, int bits, const void* sc, const void* bi);
size_t i8_total_workspace(long long M, long long N, long long K, int gs, int bits);
int launch_qmv_i8(const uint16_t* x, const uint32_t* w, const uint16_t* sc, const uint16_t* bi, uint16_t* y, int M,
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st);
}  // namespace qmm_host

extern "C" int qmm_quantized_matmul_noalloc(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                            void* y, int64_t M, int64_t N, int64_t K, int group_size, int bits,
                                            int dtype, void* stream) {
    using namespace qmm_host;
    if (dtype != QMM_BF16 && dtype != QMM_F16) {
        set_error("dtype %d: activations must be bf16 or fp16", dtype);
        return QMM_EUNSUPPORTED;
    }
    if ((bits != 4 && bits != 8) || (group_size != 32 && group_size != 64 && group_size != 128)) {
        set_error("bits=%d group_size=%d: 4/8-bit codes, groups of 32/64/128", bits, group_size);
        return QMM_EUNSUPPORTED;
    }
    if (M < 1 || M > 16) {
        set_error("noalloc: M=%lld; this entry point serves the decode kernel (1 <= M <= 16)", (long long)M);
        return QMM_EUNSUPPORTED;
    }
    if (N <= 0 || K <= 0 || K % group_size || N > (1LL << 30) || K > (1LL << 30)) {
        set_error("noalloc: bad shape N=%lld K=%lld", (long long)N, (long long)K);
        return QMM_EINVAL;
    }
    if (!x || !w || !scales || !biases || !y) {
        set_error("null pointer argument");
        return QMM_EINVAL;
    }
    if (((uintptr_t)x & 15u) || ((uintptr_t)w & 15u) || ((uintptr_t)y & 15u)) {
        set_error("x, w and y must be 16-byte aligned");
        return QMM_EINVAL;
    }
    // the same kernel choice as qmm_quantized_matmul (so the two agree bit for bit)
    const bool i8 = i8_eligible(M, N, K, group_size, bits, scales, biases);
    int rw = 0, kw = 0, kc = 1;
    if (!i8 && (qmv_cta_preferred(N, K, group_size, bits, &rw, &kw, &kc) ||
                (M > 8 && qmv_cta_preferred_wide(N, K, group_size, bits, &rw, &kw)))) {
        // the CTA-per-tile kernel reduces in shared memory: no scratch
        fire("qmv");
        qmm::QmvArgs a{};
        a.x = static_cast<const uint16_t*>(x);
        a.w = w;
        a.sc = static_cast<const uint16_t*>(scales);
        a.bi = static_cast<const uint16_t*>(biases);
        a.y = static_cast<uint16_t*>(y);
        a.M = (int)M;
        a.N = (int)N;
        a.K = (int)K;
        return launch_qmv<false>(a, bits, group_size, dtype == QMM_F16, M <= 8 ? 1 : 2, rw, kw, kc,
                                 static_cast<cudaStream_t>(stream));
    }
    const size_t need = i8 ? i8_total_workspace(M, N, K, group_size, bits) : sk_workspace(M, N, K, group_size, bits);
    if (need > kScratchBytes) {
        set_error("noalloc: N=%lld K=%lld needs %zu bytes of scratch, more than the %zu-byte built-in array; "
                  "use qmm_quantized_matmul with a workspace",
                  (long long)N, (long long)K, need, kScratchBytes);
        return QMM_EUNSUPPORTED;
    }
    void* scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the counters this call's tiles use must start at zero (16-row tiles bound them)
    size_t counters = (size_t)((N + 15) / 16) * sizeof(int);
    if (counters > kCounterBytes) counters = kCounterBytes;
    cudaError_t e = cudaMemsetAsync(scratch, 0, counters, st);
    if (e != cudaSuccess) return cuda_status(e, "noalloc: clearing the tile counters");
    fire("qmv");
    if (i8) {
        fire("qmv_i8");
        return launch_qmv_i8(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                             static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N, (int)K,
                             group_size, bits, dtype == QMM_F16, scratch, kScratchBytes, st);
    }
    return launch_qmv_sk(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                         static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N, (int)K,
                         group_size, bits, dtype == QMM_F16, scratch, kScratchBytes, st);
}
