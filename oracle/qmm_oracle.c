/*
 * qmm_oracle.c -- CPU restatement of mlxturbo's quantized-matmul hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (mlxturbo_b200/) links,
 * loads or calls this file.  It is used by tests/ as the parity checker, by
 * __graft_entry__.smoke() as the checker of one small GPU call, and by
 * bench.py's cpu_baseline / --impl reference leg as the timed CPU arm.
 *
 * Parity status: the arithmetic of the reference lives in MLX 0.32.2, which is
 * not present in this container (no Metal, no network).  What is pinned:
 *   - code unpacking and the affine dequantisation (s*q + b, bits 2..8) are
 *     checked bit-exactly against golden vectors produced by compiling the
 *     reference's own `dequantize` template (mlxturbo/kernels/_steel_flat.py,
 *     the quantized.h:483-569 excerpt) -- see oracle/ref_dequant/.
 *   - the MLX qmv_fast per-lane accumulation order (qmv_small_m.py:79-218) is
 *     restated in oracle_qmv_mlx_order(); the cross-lane simd_sum tree and the
 *     Metal compiler's FMA contraction are hardware/compiler defined and stay
 *     unpinned.
 * Matmul parity is therefore defined against the fp32 dequantise-then-matmul
 * oracle (oracle_qmm_f32), the form the reference itself uses as its fp32
 * reference (moe_verify_gather.py:923-940, bench/test_qmm_wide_shapes.py:42-48).
 *
 * Layouts (MLX affine quantisation, mlxturbo/_mlx_compat.py:37-38):
 *   w      uint32 [N, K*bits/32]  little-endian bit stream per row, value k at
 *                                 bit offset k*bits (low bits first)
 *   scales T [N, K/group_size], biases T [N, K/group_size]
 *   x      T [M, K], y [M, N]     (transpose=True, y = x @ dequant(w)^T)
 * T is bf16 (dtype code 0) or fp16 (dtype code 1); both are passed as uint16.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* 16-bit float conversions (round to nearest even)                    */
/* ------------------------------------------------------------------ */

static inline float bits_to_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

float oracle_bf16_to_f32(uint16_t h) { return bits_to_f32((uint32_t)h << 16); }

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u = f32_to_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (exp == 0) {
        if (man == 0) return bits_to_f32(sign);
        float v = ldexpf((float)man, -24);               /* subnormal */
        return sign ? -v : v;
    }
    if (exp == 31) return bits_to_f32(sign | 0x7f800000u | (man << 13));
    return bits_to_f32(sign | ((exp + 112u) << 23) | (man << 13));
}

uint16_t oracle_f32_to_f16(float f) {
    uint32_t u = f32_to_bits(f);
    uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    uint32_t a = u & 0x7fffffffu;
    if (a > 0x7f800000u) return sign | 0x7e00u;                 /* NaN */
    if (a >= 0x477ff000u) return sign | 0x7c00u;                /* overflow -> inf */
    if (a < 0x38800000u) {                                      /* subnormal / zero */
        float af = bits_to_f32(a);
        float scaled = af * 16777216.0f;                        /* 2^24: units of 2^-24 */
        float r = nearbyintf(scaled);                           /* RNE */
        return sign | (uint16_t)r;
    }
    uint32_t lsb = (a >> 13) & 1u;
    a += 0xfffu + lsb;
    return sign | (uint16_t)((a - (112u << 23)) >> 13);
}

static inline float to_f32(uint16_t h, int dtype) {
    return dtype == 0 ? oracle_bf16_to_f32(h) : oracle_f16_to_f32(h);
}
static inline uint16_t from_f32(float f, int dtype) {
    return dtype == 0 ? oracle_f32_to_bf16(f) : oracle_f32_to_f16(f);
}

void oracle_f32_to_half_array(const float* src, int64_t n, int dtype, uint16_t* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = from_f32(src[i], dtype);
}
void oracle_half_to_f32_array(const uint16_t* src, int64_t n, int dtype, float* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = to_f32(src[i], dtype);
}

/* ------------------------------------------------------------------ */
/* Code packing: value k of a row sits at bit offset k*bits of the     */
/* row's little-endian bit stream (quantized.h dequantize, restated at  */
/* mlxturbo/kernels/_steel_flat.py:1195-1256).                          */
/* ------------------------------------------------------------------ */

static inline uint32_t get_code(const uint32_t* row, int64_t k, int bits) {
    int64_t bit = k * bits;
    int64_t word = bit >> 5;
    int off = (int)(bit & 31);
    uint64_t v = row[word];
    if (off + bits > 32) v |= (uint64_t)row[word + 1] << 32;
    return (uint32_t)((v >> off) & ((1u << bits) - 1u));
}

void oracle_unpack_codes(const uint32_t* w, int64_t N, int64_t K, int bits, uint8_t* codes) {
    int64_t wpr = K * bits / 32;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) codes[n * K + k] = (uint8_t)get_code(w + n * wpr, k, bits);
}

void oracle_pack_codes(const uint8_t* codes, int64_t N, int64_t K, int bits, uint32_t* w) {
    int64_t wpr = K * bits / 32;
    memset(w, 0, (size_t)(N * wpr) * sizeof(uint32_t));
    for (int64_t n = 0; n < N; ++n) {
        uint32_t* row = w + n * wpr;
        for (int64_t k = 0; k < K; ++k) {
            uint64_t v = codes[n * K + k] & ((1u << bits) - 1u);
            int64_t bit = k * bits;
            int64_t word = bit >> 5;
            int off = (int)(bit & 31);
            row[word] |= (uint32_t)(v << off);
            if (off + bits > 32) row[word + 1] |= (uint32_t)(v >> (32 - off));
        }
    }
}

/* Affine dequantisation s*q + b in fp32 (the steel `dequantize` computes
 * float(scale)*q + float(bias) before the cast to U, _steel_flat.py:1195-1256). */
void oracle_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int dtype,
                       int64_t N, int64_t K, int group_size, int bits, float* out) {
    int64_t wpr = K * bits / 32, G = K / group_size;
    for (int64_t n = 0; n < N; ++n)
        for (int64_t k = 0; k < K; ++k) {
            float s = to_f32(scales[n * G + k / group_size], dtype);
            float b = to_f32(biases[n * G + k / group_size], dtype);
            out[n * K + k] = s * (float)get_code(w + n * wpr, k, bits) + b;
        }
}

/* ------------------------------------------------------------------ */
/* MLX affine quantisation (mx.quantize, mode="affine"): per group      */
/* min/max, a scale nudged so that 0.0 lies on the grid, codes clipped  */
/* to [0, 2^bits-1]; scales/biases cast to the weight dtype afterwards. */
/* Restates MLX 0.32.2 `affine_quantize` (not vendored; the reference   */
/* calls it via mx.quantize in rebit.py:103-121 and the reference's     */
/* host quantizer at tools/ane_quant_probe.py:34-46 shows the per-group */
/* min/max form).                                                       */
/* ------------------------------------------------------------------ */
void oracle_quantize(const float* wf, int64_t N, int64_t K, int group_size, int bits, int dtype,
                     uint32_t* wq, uint16_t* scales, uint16_t* biases) {
    int64_t G = K / group_size;
    float n_bins = (float)((1 << bits) - 1);
    uint8_t* codes = (uint8_t*)malloc((size_t)(N * K));
    for (int64_t n = 0; n < N; ++n) {
        for (int64_t g = 0; g < G; ++g) {
            const float* v = wf + n * K + g * group_size;
            float mx = v[0], mn = v[0];
            for (int i = 1; i < group_size; ++i) {
                if (v[i] > mx) mx = v[i];
                if (v[i] < mn) mn = v[i];
            }
            int mask = fabsf(mn) > fabsf(mx);
            float scale = (mx - mn) / n_bins;
            if (scale < 1e-7f) scale = 1e-7f;
            if (!mask) scale = -scale;
            float edge = mask ? mn : mx;
            float q0 = nearbyintf(edge / scale);
            float bias = 0.0f;
            if (q0 != 0.0f) {
                scale = edge / q0;
                bias = edge;
            }
            for (int i = 0; i < group_size; ++i) {
                float q = nearbyintf((v[i] - bias) / scale);
                if (q < 0.0f) q = 0.0f;
                if (q > n_bins) q = n_bins;
                codes[n * K + g * group_size + i] = (uint8_t)q;
            }
            scales[n * G + g] = from_f32(scale, dtype);
            biases[n * G + g] = from_f32(bias, dtype);
        }
    }
    oracle_pack_codes(codes, N, K, bits, wq);
    free(codes);
}

/* ------------------------------------------------------------------ */
/* fp32 dequantise-then-matmul: y[m,n] = sum_k x[m,k] * (s*q + b).      */
/* The accumulation is per group in fp32, then across groups in fp32.  */
/* OpenMP over output rows n (the CPU baseline parallelisation).        */
/* ------------------------------------------------------------------ */
/* Dequantise one group of one row into deq[0..group_size). */
static inline void deq_group(const uint32_t* row, int64_t k0, int group_size, int bits, float s, float b,
                             float* deq) {
    if (bits == 4) {
        const uint32_t* wp = row + k0 / 8;
        for (int i = 0; i < group_size; ++i) deq[i] = s * (float)((wp[i >> 3] >> (4 * (i & 7))) & 15u) + b;
    } else if (bits == 8) {
        const uint32_t* wp = row + k0 / 4;
        for (int i = 0; i < group_size; ++i) deq[i] = s * (float)((wp[i >> 2] >> (8 * (i & 3))) & 255u) + b;
    } else {
        for (int i = 0; i < group_size; ++i) deq[i] = s * (float)get_code(row, k0 + i, bits) + b;
    }
}

/* One output row block.  Per group the dot product is accumulated in 8
 * interleaved fp32 lanes (lane i%8), the lanes are added in order, and the
 * group results are added in K order -- a fixed, vectorisable fp32 order. */
static void qmm_rows(const float* xf, int64_t M, int64_t K, const uint32_t* w, const uint16_t* scales,
                     const uint16_t* biases, int dtype, int64_t n0, int64_t n1, int64_t N, int group_size,
                     int bits, float* y, float* deq) {
    int64_t wpr = K * bits / 32, G = K / group_size;
    for (int64_t n = n0; n < n1; ++n) {
        const uint32_t* row = w + n * wpr;
        for (int64_t g = 0; g < G; ++g) {
            float s = to_f32(scales[n * G + g], dtype), b = to_f32(biases[n * G + g], dtype);
            deq_group(row, g * group_size, group_size, bits, s, b, deq + g * group_size);
        }
        for (int64_t m = 0; m < M; ++m) {
            const float* xr = xf + m * K;
            float acc = 0.0f;
            for (int64_t g = 0; g < G; ++g) {
                float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                const float* d = deq + g * group_size;
                const float* xx = xr + g * group_size;
                for (int i = 0; i < group_size; i += 8)
                    for (int j = 0; j < 8; ++j) lane[j] += xx[i + j] * d[i + j];
                float part = ((lane[0] + lane[1]) + (lane[2] + lane[3])) + ((lane[4] + lane[5]) + (lane[6] + lane[7]));
                acc += part;
            }
            y[m * N + n] = acc;
        }
    }
}

void oracle_qmm_f32(const uint16_t* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                    const uint16_t* scales, const uint16_t* biases, int64_t N, int group_size, int bits,
                    float* y, int nthreads) {
    float* xf = (float*)malloc((size_t)(M * K) * sizeof(float));
    for (int64_t i = 0; i < M * K; ++i) xf[i] = to_f32(x[i], dtype);
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
    {
        int tid = omp_get_thread_num(), nt = omp_get_num_threads();
#else
    {
        int tid = 0, nt = 1;
        (void)nthreads;
#endif
        float* deq = (float*)malloc((size_t)K * sizeof(float));
        int64_t chunk = (N + nt - 1) / nt;
        int64_t n0 = tid * chunk, n1 = n0 + chunk < N ? n0 + chunk : N;
        if (n0 < n1) qmm_rows(xf, M, K, w, scales, biases, dtype, n0, n1, N, group_size, bits, y, deq);
        free(deq);
    }
    free(xf);
}

/* ------------------------------------------------------------------ */
/* MLX qmv_fast per-lane order for 4-bit (restated from the reference's */
/* bit-identical copy, mlxturbo/kernels/qmv_small_m.py:79-218):          */
/*  - lane l owns 16 contiguous K values of each 512 block;              */
/*  - x is pre-scaled (x0, x1/16, x2/256, x3/4096) and multiplied with   */
/*    the unshifted masked code (w&0x000f, w&0x00f0, ...);               */
/*  - the per-block x sum adds 4 values in T precision before widening;  */
/*  - per block res += s*acc + b*sum; then the 32 lane sums are added.   */
/* Unpinned: the simd_sum tree (summed here in lane order) and the      */
/* Metal compiler's FMA contraction (none here).                         */
/* ------------------------------------------------------------------ */
static inline float round_t(float v, int dtype) { return to_f32(from_f32(v, dtype), dtype); }

void oracle_qmv_mlx_order(const uint16_t* x, int dtype, int64_t M, int64_t K, const uint32_t* w,
                          const uint16_t* scales, const uint16_t* biases, int64_t N, uint16_t* y) {
    const int group_size = 64;
    int64_t G = K / group_size, wpr = K / 8;
    for (int64_t m = 0; m < M; ++m) {
        const uint16_t* xr = x + m * K;
        for (int64_t n = 0; n < N; ++n) {
            const uint16_t* row16 = (const uint16_t*)(w + n * wpr);
            float lane_res[32];
            for (int l = 0; l < 32; ++l) {
                float res = 0.0f;
                for (int64_t k0 = 0; k0 < K; k0 += 512) {
                    int64_t kb = k0 + 16 * l;
                    float s = to_f32(scales[n * G + kb / group_size], dtype);
                    float b = to_f32(biases[n * G + kb / group_size], dtype);
                    float acc = 0.0f, sum = 0.0f;
                    for (int i = 0; i < 4; ++i) {
                        const uint16_t* xp = xr + kb + 4 * i;
                        float t0 = to_f32(xp[0], dtype);
                        float t1 = to_f32(xp[1], dtype) / 16.0f;
                        float t2 = to_f32(xp[2], dtype) / 256.0f;
                        float t3 = to_f32(xp[3], dtype) / 4096.0f;
                        float s01 = round_t(to_f32(xp[0], dtype) + to_f32(xp[1], dtype), dtype);
                        float s012 = round_t(s01 + to_f32(xp[2], dtype), dtype);
                        float s0123 = round_t(s012 + to_f32(xp[3], dtype), dtype);
                        sum += s0123;
                        uint16_t wi = row16[kb / 4 + i];
                        float n0 = (float)(wi & 0x000f), n1 = (float)(wi & 0x00f0);
                        float n2 = (float)(wi & 0x0f00), n3 = (float)(wi & 0xf000);
                        acc += (t0 * n0 + t1 * n1 + t2 * n2 + t3 * n3);
                    }
                    res += s * acc + b * sum;
                }
                lane_res[l] = res;
            }
            float tot = 0.0f;
            for (int l = 0; l < 32; ++l) tot += lane_res[l];
            y[m * N + n] = from_f32(tot, dtype);
        }
    }
}

/* ------------------------------------------------------------------ */
/* gather_qmm: y[r] = x[lhs[r]] @ dequant(w[rhs[r]])^T                   */
/* (mx.gather_qmm with transpose=True; the reference passes rhs_indices  */
/* only, fused.py:3105-3116; lhs_indices default to the identity).      */
/* w is [E, N, K*bits/32], scales/biases [E, N, K/gs].                   */
/* ------------------------------------------------------------------ */
void oracle_gather_qmm_f32(const uint16_t* x, int dtype, int64_t x_rows, int64_t K, const uint32_t* w,
                           const uint16_t* scales, const uint16_t* biases, int64_t E, int64_t N,
                           int group_size, int bits, const int32_t* lhs, const int32_t* rhs, int64_t rows,
                           float* y, int nthreads) {
    int64_t wpe = N * (K * bits / 32), spe = N * (K / group_size);
    (void)E;
    (void)x_rows;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
#endif
    for (int64_t r = 0; r < rows; ++r) {
        int64_t xr = lhs ? lhs[r] : r;
        int64_t e = rhs[r];
        float* xf = (float*)malloc((size_t)K * sizeof(float));
        float* deq = (float*)malloc((size_t)K * sizeof(float));
        for (int64_t k = 0; k < K; ++k) xf[k] = to_f32(x[xr * K + k], dtype);
        qmm_rows(xf, 1, K, w + e * wpe, scales + e * spe, biases + e * spe, dtype, 0, N, N, group_size, bits,
                 y + r * N, deq);
        free(xf);
        free(deq);
    }
}

/* ------------------------------------------------------------------ */
/* MoE glue                                                             */
/* ------------------------------------------------------------------ */

/* Stable counting sort of expert ids: order = stable argsort(ids),
 * idx_s = ids[order], row_src = order / top_k, inv = argsort(order)
 * (the four arrays of _vendor/qwen4_exp.py:1775-1778 and fused._inv_perm,
 * produced without atomics in moe_counting_sort.py:41-80). */
void oracle_sort_rows(const uint32_t* ids, int64_t M, int64_t E, int top_k, uint32_t* order, uint32_t* idx_s,
                      uint32_t* row_src, uint32_t* inv) {
    /* ids >= E are padding rows: one extra bucket E after every expert, in
     * input order, reported with idx_s = E */
    int64_t* cur = (int64_t*)calloc((size_t)(E + 2), sizeof(int64_t));
    for (int64_t i = 0; i < M; ++i) cur[(ids[i] < (uint64_t)E ? ids[i] : E) + 1]++;
    for (int64_t e = 0; e <= E; ++e) cur[e + 1] += cur[e];
    for (int64_t i = 0; i < M; ++i) {
        int64_t pos = cur[ids[i] < (uint64_t)E ? ids[i] : E]++;
        order[pos] = (uint32_t)i;
    }
    for (int64_t s = 0; s < M; ++s) {
        const uint32_t e = ids[order[s]];
        idx_s[s] = e < (uint32_t)E ? e : (uint32_t)E;
        row_src[s] = order[s] / (uint32_t)top_k;
        inv[order[s]] = (uint32_t)s;
    }
    free(cur);
}

/* row_start[e] = first sorted row of expert e; tile_prefix[e] = tiles of the
 * experts before e, with bm-row tiles, or 16/32-row tiles chosen per expert
 * by `rows_e < mix_threshold` when mix_threshold > 0
 * (moe_grouped_gemm.py:829-855 segment_tables). */
void oracle_segment_tables(const int32_t* counts, int64_t E, int bm, int mix_threshold, int32_t* row_start,
                           int32_t* tile_prefix) {
    row_start[0] = 0;
    tile_prefix[0] = 0;
    for (int64_t e = 0; e < E; ++e) {
        int c = counts[e];
        int b = bm;
        if (mix_threshold > 0) b = c < mix_threshold ? 16 : 32;
        row_start[e + 1] = row_start[e] + c;
        tile_prefix[e + 1] = tile_prefix[e] + (c + b - 1) / b;
    }
}

/* y[t,n] = sum_k w[t*top_k+k] * out_sorted[inv[t*top_k+k], n], fp32
 * accumulation in k order, one rounding at the store
 * (mlxturbo/kernels/moe_combine.py:1-60). */
void oracle_moe_combine(const uint16_t* out_sorted, int dtype, const uint32_t* inv, const float* wts,
                        int64_t rows, int top_k, int64_t N, uint16_t* y, float* y_f32) {
    for (int64_t t = 0; t < rows; ++t)
        for (int64_t n = 0; n < N; ++n) {
            float acc = 0.0f;
            for (int k = 0; k < top_k; ++k) {
                int64_t i = t * top_k + k;
                acc += wts[i] * to_f32(out_sorted[(int64_t)inv[i] * N + n], dtype);
            }
            if (y) y[t * N + n] = from_f32(acc, dtype);
            if (y_f32) y_f32[t * N + n] = acc;
        }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
