// prefill.cu -- M > 16 quantized matmul on tensor cores (sm_100a).
#include "common.cuh"

namespace qmm_host {

int prefill_supported(int bits, int gs) {
    (void)bits;
    (void)gs;
    return 0;
}

int launch_prefill(const uint16_t*, const uint32_t*, const uint16_t*, const uint16_t*, uint16_t*, long long,
                   long long, long long, int, int, bool, cudaStream_t) {
    set_error("prefill kernel not built");
    return QMM_EUNSUPPORTED;
}

}  // namespace qmm_host
