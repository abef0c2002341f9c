// tma.cuh -- mbarrier, TMA and programmatic-dependent-launch helpers (sm_100a).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace qmm {

QMM_DEVINL uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

QMM_DEVINL void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
QMM_DEVINL void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
QMM_DEVINL void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
QMM_DEVINL void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Bounded wait for the phase of `parity` to complete.  Returns false (and sets
// *abort and *err) when the bound is hit; once *abort is set, later waits of
// the CTA return at once so the kernel drains instead of timing out repeatedly.
QMM_DEVINL bool mbar_wait_bounded(uint32_t bar, uint32_t parity, volatile int* abort, int* err) {
    for (uint32_t i = 0; i < (1u << 20); ++i) {
        if ((i & 1023u) == 1023u && *abort) return false;
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    *abort = 1;
    atomicExch(err, 1);
    return false;
}

QMM_DEVINL void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(map), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing on an mbarrier's transaction count.
QMM_DEVINL void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

QMM_DEVINL void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Programmatic dependent launch: let the next kernel of the stream start its
// independent prologue now; wait until the previous kernel's results are
// visible before touching them.  Both are no-ops without the launch attribute.
QMM_DEVINL void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
QMM_DEVINL void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace qmm

namespace qmm_host {
// 2-D tensor map (dims innermost first).  Cached by (base, dims, box, dtype,
// swizzle): the descriptor depends only on those.
int tensor_map_2d(CUtensorMap* out, CUtensorMapDataType dt, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz);
// Whether kernels should be launched with programmatic stream serialization.
bool pdl_enabled();
// Raise `func`'s dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute is per device, so the setting is remembered
// per (kernel, device) and made again for a device that has not seen it;
// thread-safe.  Returns a qmm_status.
int ensure_smem_limit(const void* func, int bytes, const char* what);
}  // namespace qmm_host
