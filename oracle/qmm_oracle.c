/*
 * CPU oracle for the small-M affine-quantized matmul (TEST INFRASTRUCTURE ONLY).
 *
 * This file is the checker, never the product: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it.  The CUDA library
 * (libdflashcuda.so) never links or calls it.
 *
 * What it restates (all citations relative to the random1st/dflash-swift tree):
 *
 *   - MLX packed layout consumed by the reference kernel,
 *     Sources/DFlashKit/SmallMQuantizedMatmul.swift:55-71:
 *       4-bit: word (n, kw) of a [N, K/8] uint32 matrix holds k = 8*kw .. 8*kw+7,
 *              value t of the word is (p >> 4t) & 15 (low nibble first).
 *       8-bit: word (n, kw) of a [N, K/4] matrix holds k = 4*kw .. 4*kw+3,
 *              value t is (p >> 8t) & 255.
 *   - Scale/bias indexing, SmallMQuantizedMatmul.swift:127-129: one bf16 pair per
 *     group of `group` consecutive k in row n, at [n * (K/group) + k/group].
 *   - Dequantisation w = q * s + b, two flavours:
 *       QMM_FLAVOUR_EXACT  : fp32 q*s+b kept exact (stock quantizedMatmul semantics,
 *                            the call SmallMQuantizedLinear stands in for,
 *                            SmallMQuantizedMatmul.swift:254-292);
 *       QMM_FLAVOUR_BF16DQ : bf16((float)q * s + b), the reference Metal kernel's
 *                            rounding of each dequantised weight,
 *                            SmallMQuantizedMatmul.swift:59,61,69.
 *     Accumulation is fp64 in both, so the oracle is more accurate than either GPU.
 *   - The affine quantizer that produces those tensors (MLX `quantize`, used by
 *     `QuantizedLinear(weight:bias:groupSize:bits:)` in
 *     Tests/DFlashKitTests/SmallMQuantizedMatmulTests.swift:54): restated from MLX's
 *     published affine_quantize (mlx-swift 0.31.6, un-vendored dependency pinned in
 *     Package.resolved at rev 0bb916c6).  The reference tree holds no vectors for it,
 *     so quantizer parity with MLX is UNPINNED; matmul parity does not depend on it
 *     because oracle and kernel consume the same packed tensors.
 *
 * Pinning: the reference's own Metal kernel text is compiled here on the CPU by
 * oracle/ref_metal (outputs in oracle/_ref/), and tests/test_oracle.py checks this
 * oracle's BF16DQ flavour against it; tests/golden/ holds vectors produced by that
 * compiled reference kernel.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QMM_FLAVOUR_EXACT 0
#define QMM_FLAVOUR_BF16DQ 1

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* IEEE round-to-nearest-even float -> bfloat16 (NaN kept quiet). */
static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

uint16_t oracle_f32_to_bf16(float f) { return f32_to_bf16(f); }
float oracle_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }

/* q value (unsigned integer code) of element (n, k). */
static inline uint32_t code_at(const uint32_t* w, int n, int k, int K, int bits) {
    const int per_word = 32 / bits;
    const uint32_t word = w[(size_t)n * (size_t)(K / per_word) + (size_t)(k / per_word)];
    const int t = k % per_word;
    return (word >> (bits * t)) & ((1u << bits) - 1u);
}

/*
 * MLX affine quantisation of a row-major fp32 [N, K] matrix.
 * Per group of `group` values: scale = (max-min)/(2^bits-1) with the sign and
 * zero-point refinement of MLX (the edge value of larger magnitude is made exactly
 * representable), bias = that edge, q = clamp(round((w-b)/s), 0, 2^bits-1).
 * Scales and biases are rounded to bf16 at the end; q is computed from the fp32
 * scale/bias, as MLX does before casting them to the weight dtype.
 * refine=0 gives the plain min/max quantizer (scale=(max-min)/n_bins, bias=min).
 */
void oracle_quantize_affine(const float* wf, int N, int K, int group, int bits, int refine,
                            uint32_t* wq, uint16_t* scales, uint16_t* biases) {
    const int per_word = 32 / bits;
    const int n_bins = (1 << bits) - 1;
    const int groups = K / group;
    memset(wq, 0, sizeof(uint32_t) * (size_t)N * (size_t)(K / per_word));
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int g = 0; g < groups; ++g) {
            const float* src = wf + (size_t)n * K + (size_t)g * group;
            float wmax = src[0], wmin = src[0];
            for (int i = 1; i < group; ++i) {
                if (src[i] > wmax) wmax = src[i];
                if (src[i] < wmin) wmin = src[i];
            }
            float scale, bias;
            if (refine) {
                const int mask = fabsf(wmin) > fabsf(wmax);
                scale = fmaxf((wmax - wmin) / (float)n_bins, 1e-7f);
                scale = mask ? scale : -scale;
                const float edge = mask ? wmin : wmax;
                const float q0 = rintf(edge / scale);
                if (q0 != 0.0f) scale = edge / q0;
                bias = (q0 == 0.0f) ? 0.0f : edge;
            } else {
                scale = fmaxf((wmax - wmin) / (float)n_bins, 1e-7f);
                bias = wmin;
            }
            scales[(size_t)n * groups + g] = f32_to_bf16(scale);
            biases[(size_t)n * groups + g] = f32_to_bf16(bias);
            for (int i = 0; i < group; ++i) {
                float q = rintf((src[i] - bias) / scale);
                if (q < 0.0f) q = 0.0f;
                if (q > (float)n_bins) q = (float)n_bins;
                const int k = g * group + i;
                wq[(size_t)n * (size_t)(K / per_word) + (size_t)(k / per_word)] |=
                    ((uint32_t)q) << (bits * (k % per_word));
            }
        }
    }
}

/* Dequantise to fp32 [N, K] (flavour as above; BF16DQ values are exactly bf16). */
void oracle_dequantize(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int N,
                       int K, int group, int bits, int flavour, float* out) {
    const int groups = K / group;
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        for (int k = 0; k < K; ++k) {
            const float s = bf16_to_f32(scales[(size_t)n * groups + k / group]);
            const float b = bf16_to_f32(biases[(size_t)n * groups + k / group]);
            const float q = (float)code_at(w, n, k, K, bits);
            float v = q * s + b;
            if (flavour == QMM_FLAVOUR_BF16DQ) v = bf16_to_f32(f32_to_bf16(v));
            out[(size_t)n * K + k] = v;
        }
    }
}

/*
 * y[m, n] = sum_k x[m, k] * deq(w)[n, k]   (transpose=true semantics), fp64 result.
 * x is bf16 [M, K] row-major; y is fp64 [M, N] row-major.
 * For EXACT the dequantised weight q*s+b is formed in fp64 (exact for bf16 s, b and
 * q < 2^8), i.e. the mathematically exact dequantisation.
 */
void oracle_qmm_f64(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                    const uint16_t* biases, int M, int N, int K, int group, int bits, int flavour,
                    double* y) {
    const int groups = K / group;
    double* xd = (double*)malloc(sizeof(double) * (size_t)M * K);
    for (size_t i = 0; i < (size_t)M * K; ++i) xd[i] = (double)bf16_to_f32(x[i]);
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; ++n) {
        double acc[16 * 4];
        double* a = (M <= 64) ? acc : NULL;
        double* heap = NULL;
        if (!a) a = heap = (double*)calloc((size_t)M, sizeof(double));
        for (int m = 0; m < M; ++m) a[m] = 0.0;
        for (int k = 0; k < K; ++k) {
            const float s = bf16_to_f32(scales[(size_t)n * groups + k / group]);
            const float b = bf16_to_f32(biases[(size_t)n * groups + k / group]);
            const uint32_t q = code_at(w, n, k, K, bits);
            double wv;
            if (flavour == QMM_FLAVOUR_BF16DQ)
                wv = (double)bf16_to_f32(f32_to_bf16((float)q * s + b));
            else
                wv = (double)q * (double)s + (double)b;
            for (int m = 0; m < M; ++m) a[m] += xd[(size_t)m * K + k] * wv;
        }
        for (int m = 0; m < M; ++m) y[(size_t)m * N + n] = a[m];
        free(heap);
    }
    free(xd);
}

/*
 * The timed CPU restatement (the cpu_baseline / --impl reference arm): dequantise on
 * the fly per group, fp32 accumulate, bf16 out, rows n split over OpenMP threads.
 * Semantics EXACT (fp32 q*s+b, SmallMQuantizedMatmul.swift:59 without the bf16 round).
 * Returns the number of threads used.
 */
int oracle_qmm_bf16_fp32acc(const uint16_t* x, const uint32_t* w, const uint16_t* scales,
                            const uint16_t* biases, int M, int N, int K, int group, int bits,
                            int n_begin, int n_end, int threads, uint16_t* y) {
    const int groups = K / group;
    const int per_word = 32 / bits;
    const uint32_t mask = (1u << bits) - 1u;
    float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
    for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = bf16_to_f32(x[i]);
    int used = 1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
    {
#ifdef _OPENMP
#pragma omp single
        used = omp_get_num_threads();
#endif
        float wrow[128];
#pragma omp for schedule(static)
        for (int n = n_begin; n < n_end; ++n) {
            float acc[16];
            for (int m = 0; m < M && m < 16; ++m) acc[m] = 0.0f;
            const uint32_t* wr = w + (size_t)n * (size_t)(K / per_word);
            for (int g = 0; g < groups; ++g) {
                const float s = bf16_to_f32(scales[(size_t)n * groups + g]);
                const float b = bf16_to_f32(biases[(size_t)n * groups + g]);
                for (int i = 0; i < group; ++i) {
                    const int k = g * group + i;
                    const uint32_t q = (wr[k / per_word] >> (bits * (k % per_word))) & mask;
                    wrow[i] = (float)q * s + b;
                }
                for (int m = 0; m < M && m < 16; ++m) {
                    const float* xr = xf + (size_t)m * K + (size_t)g * group;
                    float sum = 0.0f;
                    for (int i = 0; i < group; ++i) sum += xr[i] * wrow[i];
                    acc[m] += sum;
                }
            }
            for (int m = 0; m < M && m < 16; ++m) y[(size_t)m * N + n] = f32_to_bf16(acc[m]);
        }
    }
    free(xf);
    return used;
}
