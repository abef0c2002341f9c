// common.cuh -- shared device helpers for the sm_100a quantized-matmul kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mlxturbo_b200.h"

#define QMM_DEVINL __device__ __forceinline__

namespace qmm {

// ---------------------------------------------------------------------------
// 16-bit float traits.  Activations, scales, biases and outputs share one
// dtype T (bf16 or fp16); kernels treat them as raw uint16 bit patterns.
// ---------------------------------------------------------------------------
template <bool F16>
struct Half;

template <>
struct Half<false> {  // bf16
    // bf16x2 holding (128 + q_lo, 128 + q_hi) when OR-ed onto two 4-bit codes
    // placed at bits 0..3 and 16..19: exponent 2^7, mantissa step 1.
    static constexpr uint32_t kMagic = 0x43004300u;
    static constexpr float kOffset = 128.0f;
    static constexpr uint32_t kOne2 = 0x3F803F80u;  // (1.0, 1.0)
    static QMM_DEVINL float to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
    // low / high element of a packed pair, widened to f32
    static QMM_DEVINL float lo_f32(uint32_t w) { return __uint_as_float(w << 16); }
    static QMM_DEVINL float hi_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
    static QMM_DEVINL uint16_t from_f32(float f) {
        uint16_t r;
        asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
        return r;
    }
    static QMM_DEVINL uint32_t pack2(float lo, float hi) {
        uint32_t r;
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        return r;
    }
};

template <>
struct Half<true> {  // fp16
    // f16x2 (1024 + q): exponent 2^10, mantissa step 1.
    static constexpr uint32_t kMagic = 0x64006400u;
    static constexpr float kOffset = 1024.0f;
    static constexpr uint32_t kOne2 = 0x3C003C00u;
    static QMM_DEVINL float to_f32(uint16_t h) {
        float f;
        asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
        return f;
    }
    static QMM_DEVINL float lo_f32(uint32_t w) { return to_f32((uint16_t)(w & 0xFFFFu)); }
    static QMM_DEVINL float hi_f32(uint32_t w) { return to_f32((uint16_t)(w >> 16)); }
    static QMM_DEVINL uint16_t from_f32(float f) {
        uint16_t r;
        asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(f));
        return r;
    }
    static QMM_DEVINL uint32_t pack2(float lo, float hi) {
        uint32_t r;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        return r;
    }
};

// (a & b) | c in one LOP3.
QMM_DEVINL uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

QMM_DEVINL uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// D = A(16x16) * B(16x8) + C, fp32 accumulate, A/B bf16 or fp16.
template <bool F16>
QMM_DEVINL void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const float (&c)[4]);

// Not volatile: the compiler may interleave independent accumulation chains
// (warp MMA latency is long; throughput needs several chains in flight).
template <>
QMM_DEVINL void mma16816<false>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                const float (&c)[4]) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

template <>
QMM_DEVINL void mma16816<true>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                               const float (&c)[4]) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
          "f"(c[3]));
}

// Streaming loads of packed weights: read once, keep out of L1.
QMM_DEVINL uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
QMM_DEVINL uint2 ldg_stream_v2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
QMM_DEVINL uint32_t ldg_stream_u32(const void* p) {
    uint32_t r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
// Coherent loads of data that earlier work of the stream writes (activations,
// segment tables, sorted-row maps, a prep kernel's output).  Under
// programmatic dependent launch a kernel starts while its predecessor still
// runs, so such data is read only after griddepcontrol.wait and never through
// the non-coherent read-only path, whose contract is that the data does not
// change while the kernel runs.
QMM_DEVINL uint4 ld_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
template <typename T>
QMM_DEVINL T ld_dep(const T* p) {
    return *reinterpret_cast<const volatile T*>(p);
}
QMM_DEVINL int4 ld_dep(const int4* p) {
    int4 r;
    asm volatile("ld.global.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
QMM_DEVINL uint2 ld_dep(const uint2* p) {
    uint2 r;
    asm volatile("ld.global.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
QMM_DEVINL float2 ld_dep(const float2* p) {
    float2 r;
    asm volatile("ld.global.v2.f32 {%0,%1}, [%2];" : "=f"(r.x), "=f"(r.y) : "l"(p));
    return r;
}
// Read-only loads (weights' scales and biases: inputs no kernel writes while
// the call runs; re-read by many warps).
QMM_DEVINL uint4 ldg_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
QMM_DEVINL uint16_t ldg_u16(const void* p) {
    uint16_t r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

}  // namespace qmm

// Host-side helpers shared by the translation units.
namespace qmm_host {
void set_error(const char* fmt, ...);
void clear_error();
int cuda_status(cudaError_t e, const char* what);
void fire(const char* name);
bool aligned16(const void* p);
int check_quant(int64_t N, int64_t K, int group_size, int bits, int dtype);
int check_dense_pointers(const void* x, const void* w, const void* scales, const void* biases, const void* y);

// One call of the decode-width MoE block kernel (moe_decode.cu): the
// interleaved gate/up bank [E, 2I, H], the down bank [E, H, I], T tokens of
// top_k pairs, the workspace (barrier counter, then the pairs' SwiGLU rows).
struct MoeDecodeCall {
    const void* x;
    const int32_t* ids;
    const float* wts;
    const uint32_t* guw;
    const void* gus;
    const void* gub;
    const uint32_t* dnw;
    const void* dns;
    const void* dnb;
    void* y;
    int T, top_k, E, H, I, gs, bits, dtype;
    void* ws;
    cudaStream_t st;
};
int launch_moe_glu_decode(const MoeDecodeCall& c);
int moe_decode_supported(long long T, long long top_k, long long E, long long H, long long I, int gs, int bits);
size_t moe_decode_workspace(long long T, long long top_k, long long I);
int moe_decode_device_error(int reset);
}  // namespace qmm_host
