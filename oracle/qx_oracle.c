/*
 * CPU oracle (plain C + OpenMP) for the W4A16-LoRA GEMV and the ring-buffer
 * index math.  TEST INFRASTRUCTURE ONLY: it is the checker in tests/ and the
 * timed CPU baseline in bench.py; the product library never links it.
 *
 * Algorithm followed (paths relative to the QExtract-Infer project root):
 *   - nibble i of qweight[pr, n] is W_q[8*pr + i, n]
 *     (csrc/include/quantize_utils.h:5-8, csrc/kernels/w4a16_lora_gemv.cu:179-189);
 *   - group(k) = k / group_size (w4a16_lora_gemv.cu:181);
 *   - W = fp16((q - z) * s) computed in fp32, rounded once
 *     (tests/test_w4a16_gemv.py:68-90);
 *   - y = fp16(x.W + (alpha / rank) * (x.A).B) in fp32
 *     (tests/test_w4a16_gemv.py:178-186, w4a16_lora_gemv.cu:214-225);
 *   - ring write slot / logical order / valid length
 *     (qextract/kv_cache.py:114-152, csrc/kv_cache/ring_buffer.cu:115-123,143-209).
 *
 * fp16 <-> fp32 conversions are written here from the IEEE 754 binary16
 * definition (round to nearest, ties to even).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float qxo_h2f(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, x;
    float f;
    if (e == 0) {
        f = (float)m * (1.0f / 16777216.0f); /* m * 2^-24, exact */
        memcpy(&x, &f, 4);
        x |= sign;
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    memcpy(&f, &x, 4);
    return f;
}

uint16_t qxo_f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t a = x & 0x7fffffffu;
    if (a >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u));
    if (a >= 0x477ff000u) /* >= 65520 rounds to inf */
        return (uint16_t)(sign | 0x7c00u);
    if (a < 0x38800000u) { /* below 2^-14: binary16 subnormal or zero */
        uint32_t e = a >> 23;
        if (e < 102u) return (uint16_t)sign;
        uint32_t m = (a & 0x7fffffu) | 0x800000u;
        uint32_t sh = 126u - e; /* 14 .. 24 */
        uint32_t n = m >> sh, rem = m & ((1u << sh) - 1u), hb = 1u << (sh - 1u);
        if (rem > hb || (rem == hb && (n & 1u))) n++;
        return (uint16_t)(sign | n);
    }
    uint32_t r = a + 0xfffu + ((a >> 13) & 1u);
    return (uint16_t)(sign | ((r - 0x38000000u) >> 13));
}

static inline float round_h(float f) { return qxo_h2f(qxo_f2h(f)); }

/* Zero point of (group g, column n).  packed: GPTQ qzeros int32 [G, N/8]
 * (nibble n % 8 of word n / 8) plus zero_offset; else fp16 [G, N]. */
static inline float zero_at(const void *zeros, int packed, int zero_offset,
                            int g, int n, int N) {
    if (packed) {
        const uint32_t *z = (const uint32_t *)zeros;
        uint32_t w = z[(size_t)g * (N / 8) + n / 8];
        return (float)(((w >> (4 * (n % 8))) & 0xfu) + (uint32_t)zero_offset);
    }
    return qxo_h2f(((const uint16_t *)zeros)[(size_t)g * N + n]);
}

/* y[M, N] (fp16) and optionally y_f32[M, N] (pre-rounding).  rank == 0 or
 * A == NULL disables the LoRA term.  nthreads <= 0 uses the OpenMP default.
 * Returns 0, or -1 on a shape error. */
int qxo_w4a16_lora_gemv(const uint16_t *x, const int32_t *qweight,
                        const uint16_t *scales, const void *zeros, int zeros_packed,
                        int zero_offset, const uint16_t *A, const uint16_t *B,
                        uint16_t *y, float *y_f32, int M, int K, int N, int rank,
                        int group_size, float lora_alpha, int nthreads) {
    if (M <= 0 || K <= 0 || N <= 0 || K % 8 || group_size <= 0 || K % group_size)
        return -1;
    if (zeros_packed && N % 8) return -1;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
    const int use_lora = (rank > 0 && A && B);
    float *xf = (float *)malloc(sizeof(float) * (size_t)M * K);
    float *h = (float *)calloc((size_t)M * (rank > 0 ? rank : 1), sizeof(float));
    if (!xf || !h) { free(xf); free(h); return -1; }
    for (size_t i = 0; i < (size_t)M * K; i++) xf[i] = qxo_h2f(x[i]);

    if (use_lora) { /* h = x . A, fp32 */
        for (int m = 0; m < M; m++)
            for (int k = 0; k < K; k++) {
                float xv = xf[(size_t)m * K + k];
                const uint16_t *arow = A + (size_t)k * rank;
                for (int r = 0; r < rank; r++) h[(size_t)m * rank + r] += xv * qxo_h2f(arow[r]);
            }
    }
    const float scaling = use_lora ? lora_alpha / (float)rank : 0.0f;
    const int NB = 64; /* columns per task */
    const int nblocks = (N + NB - 1) / NB;

#pragma omp parallel for schedule(static)
    for (int b = 0; b < nblocks; b++) {
        int n0 = b * NB, n1 = n0 + NB < N ? n0 + NB : N, w = n1 - n0;
        float acc[64 * 8];
        float wcol[8 * 64];
        for (int m0 = 0; m0 < M; m0 += 8) {
            int mc = M - m0 < 8 ? M - m0 : 8;
            memset(acc, 0, sizeof(acc));
            for (int pr = 0; pr < K / 8; pr++) {
                int g = (pr * 8) / group_size;
                for (int j = 0; j < w; j++) {
                    int n = n0 + j;
                    uint32_t word = (uint32_t)qweight[(size_t)pr * N + n];
                    float s = qxo_h2f(scales[(size_t)g * N + n]);
                    float z = zero_at(zeros, zeros_packed, zero_offset, g, n, N);
                    for (int i = 0; i < 8; i++)
                        wcol[i * 64 + j] = round_h(((float)((word >> (4 * i)) & 0xfu) - z) * s);
                }
                for (int mm = 0; mm < mc; mm++) {
                    const float *xr = xf + (size_t)(m0 + mm) * K + pr * 8;
                    float *ar = acc + mm * 64;
                    for (int i = 0; i < 8; i++) {
                        float xv = xr[i];
                        const float *wr = wcol + i * 64;
                        for (int j = 0; j < w; j++) ar[j] += xv * wr[j];
                    }
                }
            }
            for (int mm = 0; mm < mc; mm++) {
                int m = m0 + mm;
                for (int j = 0; j < w; j++) {
                    int n = n0 + j;
                    float lora = 0.0f;
                    if (use_lora)
                        for (int r = 0; r < rank; r++)
                            lora += h[(size_t)m * rank + r] * qxo_h2f(B[(size_t)r * N + n]);
                    float v = acc[mm * 64 + j] + scaling * lora;
                    if (y_f32) y_f32[(size_t)m * N + n] = v;
                    if (y) y[(size_t)m * N + n] = qxo_f2h(v);
                }
            }
        }
    }
    free(xf);
    free(h);
    return 0;
}

/* W[K, N] = fp16((q - z) * s) in fp32, rounded once (tests/test_w4a16_gemv.py:68-90),
 * the dequantised weight of the GEMV above, written out for the large checks.
 * Returns 0, or -1 on a shape error. */
int qxo_dequantize(const int32_t *qweight, const uint16_t *scales, const void *zeros,
                   int zeros_packed, int zero_offset, uint16_t *W, int K, int N,
                   int group_size, int nthreads) {
    if (K <= 0 || N <= 0 || K % 8 || group_size <= 0 || K % group_size) return -1;
    if (zeros_packed && N % 8) return -1;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
#pragma omp parallel for schedule(static)
    for (int pr = 0; pr < K / 8; pr++) {
        int g = (pr * 8) / group_size;
        for (int n = 0; n < N; n++) {
            uint32_t word = (uint32_t)qweight[(size_t)pr * N + n];
            float s = qxo_h2f(scales[(size_t)g * N + n]);
            float z = zero_at(zeros, zeros_packed, zero_offset, g, n, N);
            for (int i = 0; i < 8; i++)
                W[(size_t)(pr * 8 + i) * N + n] = qxo_f2h(((float)((word >> (4 * i)) & 0xfu) - z) * s);
        }
    }
    return 0;
}

/* Ring-buffer index math (qextract/kv_cache.py:114-152). */
int64_t qxo_ring_write_pos(int64_t count, int sink, int window) {
    if (count < sink) return count;
    return sink + (count - sink) % window;
}

int64_t qxo_ring_valid_length(int64_t count, int sink, int window) {
    if (count <= sink) return count;
    int64_t f = count - sink;
    return sink + (f < window ? f : window);
}

/* Writes valid_length(count) slot indices in logical order; returns that length. */
int64_t qxo_ring_indices(int64_t count, int sink, int window, int32_t *out) {
    int64_t ns = count < sink ? count : sink, n = 0;
    for (int64_t i = 0; i < ns; i++) out[n++] = (int32_t)i;
    if (count > sink) {
        int64_t f = count - sink;
        int64_t filled = f < window ? f : window;
        int64_t start = (f <= window) ? 0 : f % window;
        for (int64_t i = 0; i < filled; i++) out[n++] = (int32_t)(sink + (start + i) % window);
    }
    return n;
}
