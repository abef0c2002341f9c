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
// remembers it.  That first call also clears the array, with a memset on the
// caller's stream (so the clear is ordered before the call's own kernels on
// any stream, blocking or not); it should come before any stream capture on
// that device.
//
// All calls on a device share the array and it keeps the last call's
// contents.  The stream-K kernel's tile counters must be zero when a call
// starts: each call that runs that kernel clears the counters it will use on
// its stream first (the kernel leaves them zero again).  The integer-MMA
// kernel tags its partial sums with a per-call epoch kept in the array, so an
// earlier call's partials never read as this call's.  Two calls that overlap
// on the GPU -- different streams, or different host threads without
// ordering -- race on the array and give wrong results.
//
// Kernel choice: the same as qmm_quantized_matmul given a workspace of
// kScratchBytes.  Every decode shape of the benchmarked models fits; a matrix
// of >= 12 MiB of codes with K above about 200k would need more than the
// integer-MMA kernel's share of the array and runs on the CTA-per-tile or
// stream-K kernel instead (results then match qmm_quantized_matmul within the
// usual bf16/fp16 tolerance, not bit for bit).

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

// Device address of the scratch array on the current device (set up on the
// first use, which also clears the array on `st`).
int scratch_for_current_device(void** out, cudaStream_t st) {
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
        e = cudaMemsetAsync(p, 0, kScratchBytes, st);
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
                  int N, int K, int gs, int bits, bool f16, void* ws, size_t ws_bytes, cudaStream_t st,
                  unsigned long long* amax = nullptr, long long n_offset = 0);
}  // namespace qmm_host

extern "C" int qmm_quantized_matmul_noalloc(const void* x, const uint32_t* w, const void* scales, const void* biases,
                                            void* y, int64_t M, int64_t N, int64_t K, int group_size, int bits,
                                            int dtype, void* stream) {
    using namespace qmm_host;
    clear_error();
    int rc = check_quant(N, K, group_size, bits, dtype);
    if (rc) return rc;
    if (M < 0) {
        set_error("noalloc: M=%lld < 0", (long long)M);
        return QMM_EINVAL;
    }
    if (M == 0) return QMM_OK;
    if (M > 16) {
        set_error("noalloc: M=%lld; this entry point serves the decode kernels (1 <= M <= 16)", (long long)M);
        return QMM_EUNSUPPORTED;
    }
    rc = check_dense_pointers(x, w, scales, biases, y);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the same kernel choice as qmm_quantized_matmul with a kScratchBytes workspace
    const bool i8 = i8_eligible(M, N, K, group_size, bits, scales, biases) &&
                    i8_total_workspace(M, N, K, group_size, bits) <= kScratchBytes;
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
        return launch_qmv<false>(a, bits, group_size, dtype == QMM_F16, M <= 8 ? 1 : 2, rw, kw, kc, st);
    }
    if (!i8 && sk_workspace(M, N, K, group_size, bits) > kScratchBytes) {
        set_error("noalloc: N=%lld K=%lld needs %zu bytes of scratch, more than the %zu-byte built-in array; "
                  "use qmm_quantized_matmul with a workspace",
                  (long long)N, (long long)K, sk_workspace(M, N, K, group_size, bits), kScratchBytes);
        return QMM_EUNSUPPORTED;
    }
    void* scratch = nullptr;
    rc = scratch_for_current_device(&scratch, st);
    if (rc) return rc;
    fire("qmv");
    if (i8) {
        fire("qmv_i8");
        return launch_qmv_i8(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                             static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N, (int)K,
                             group_size, bits, dtype == QMM_F16, scratch, kScratchBytes, st);
    }
    // the stream-K kernel's tile counters this call uses must start at zero (16-row tiles bound them)
    size_t counters = (size_t)((N + 15) / 16) * sizeof(int);
    if (counters > kCounterBytes) counters = kCounterBytes;
    cudaError_t e = cudaMemsetAsync(scratch, 0, counters, st);
    if (e != cudaSuccess) return cuda_status(e, "noalloc: clearing the tile counters");
    return launch_qmv_sk(static_cast<const uint16_t*>(x), w, static_cast<const uint16_t*>(scales),
                         static_cast<const uint16_t*>(biases), static_cast<uint16_t*>(y), (int)M, (int)N, (int)K,
                         group_size, bits, dtype == QMM_F16, scratch, kScratchBytes, st);
}
