// tmap.cu -- host side of TMA: cuTensorMapEncodeTiled through the runtime's
// driver entry point (no libcuda link), with a small descriptor cache so a
// decode step does not re-encode the same weight matrix on every call.

#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "tma.cuh"

namespace qmm_host {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::mutex g_mu;

struct MapKey {
    const void* base;
    uint64_t inner, outer, row_bytes;
    uint32_t box_inner, box_outer;
    int dt, swz;
};

// hashed: a lookup probes at most kProbe slots, whatever the number of maps
// encoded so far (a linear scan of a full table cost microseconds per call)
static constexpr int kCache = 1024, kProbe = 4;
static MapKey g_keys[kCache];
static CUtensorMap g_maps[kCache];
static bool g_valid[kCache];

static uint32_t key_hash(const MapKey& k) {
    uint64_t h = 1469598103934665603ull;
    const uint64_t words[6] = {(uint64_t)(uintptr_t)k.base, k.inner, k.outer, k.row_bytes,
                               ((uint64_t)k.box_inner << 32) | k.box_outer, ((uint64_t)(uint32_t)k.dt << 32) | (uint32_t)k.swz};
    for (uint64_t w : words) {
        h ^= w;
        h *= 1099511628211ull;
        h ^= h >> 29;
    }
    return (uint32_t)h;
}

static int get_encode() {
    if (g_encode) return QMM_OK;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        set_error("cuTensorMapEncodeTiled unavailable");
        return QMM_ECUDA;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return QMM_OK;
}

int tensor_map_2d(CUtensorMap* out, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
    const MapKey key{base, inner, outer, row_bytes, box_inner, box_outer, (int)dt, (int)swz};
    const uint32_t h0 = key_hash(key) & (kCache - 1);
    std::lock_guard<std::mutex> lock(g_mu);
    for (int i = 0; i < kProbe; ++i) {
        const uint32_t j = (h0 + i) & (kCache - 1);
        if (g_valid[j] && memcmp(&g_keys[j], &key, sizeof(MapKey)) == 0) {
            *out = g_maps[j];
            return QMM_OK;
        }
    }
    int rc = get_encode();
    if (rc) return rc;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(out, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return QMM_ECUDA;
    }
    int slot = (int)h0;  // a free probe slot, else the first (evicted)
    for (int i = 0; i < kProbe; ++i) {
        const uint32_t j = (h0 + i) & (kCache - 1);
        if (!g_valid[j]) {
            slot = (int)j;
            break;
        }
    }
    memcpy(&g_keys[slot], &key, sizeof(MapKey));
    g_maps[slot] = *out;
    g_valid[slot] = true;
    return QMM_OK;
}

// (kernel, device) -> dynamic shared-memory limit already set.  A fixed table:
// a process launches a few dozen kernel instantiations on a few devices.
namespace {
struct SmemLimit {
    const void* func;
    int dev, bytes;
};
constexpr int kSmemLimits = 512;
SmemLimit g_limits[kSmemLimits];
int g_nlimits = 0;
std::mutex g_limits_mu;
}  // namespace

int ensure_smem_limit(const void* func, int bytes, const char* what) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, what);
    std::lock_guard<std::mutex> lock(g_limits_mu);
    int slot = -1;
    for (int i = 0; i < g_nlimits; ++i)
        if (g_limits[i].func == func && g_limits[i].dev == dev) {
            if (g_limits[i].bytes >= bytes) return QMM_OK;
            slot = i;
            break;
        }
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return cuda_status(e, what);
    if (slot < 0 && g_nlimits < kSmemLimits) slot = g_nlimits++;
    if (slot >= 0) g_limits[slot] = SmemLimit{func, dev, bytes};  // a full table only re-sets the attribute
    return QMM_OK;
}

bool pdl_enabled() {
    static int v = -1;
    if (v < 0) {
        const char* e = getenv("QMM_PDL");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v == 1;
}

}  // namespace qmm_host
