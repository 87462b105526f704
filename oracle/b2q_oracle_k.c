/*
 * b2q_oracle_k.c -- CPU restatement of ggml's Q4_K weights against Q8_K
 * activations (test infrastructure only).  Q4_K is the shipped 4-bit format of
 * the reference's models (cpp_ggml/models/MODEL_CARD.md:54-74); ggml v0.21.0's
 * CPU backend runs its mul_mat with src1 quantized to Q8_K.
 *
 * block_q4_K, 256 values, 144 bytes: fp16 d, fp16 dmin, 12 bytes of 6-bit
 * sub-block scales and mins, 128 bytes of 4-bit quants.  Sub-block j (32
 * values) has scale sc_j and min m_j; value = d*sc_j*q - dmin*m_j, q in 0..15.
 * Quants: 64-value group g holds bytes qs[32g .. 32g+31]; their low nibbles are
 * values 64g..64g+31 (sub-block 2g), the high nibbles 64g+32..64g+63.
 * Scale/min unpacking: j < 4: sc = s[j] & 63, m = s[j+4] & 63; j >= 4:
 * sc = (s[j+4] & 15) | ((s[j-4] >> 6) << 4), m = (s[j+4] >> 4) | ((s[j] >> 6) << 4).
 * (Pinned against gguf-py 0.19.0's Q4_K dequantizer in tests/test_oracle.py.)
 *
 * block_q8_K, 256 values, 292 bytes: fp32 d, int8 qs[256], int16 bsums[16]
 * (sums of 16 consecutive quants).  Quantizer (ggml's reference): the value
 * with the largest |x| (first in scan order) is `max`; all zero -> d = 0 and
 * zero quants; else iscale = -127/max, q = min(127, round-half-even(iscale*x)),
 * d = 1/iscale.  Unpinned: no Q8_K vectors exist in the reference or gguf-py.
 *
 * Dot (ggml's generic form): per super-block the exact int32 sums
 *   aux[l] = sum over sub-blocks j and positions p = 32j + 8g + l of sc_j*q4*q8,
 *   sumi   = sum over the 16 bsums of bsum * m_(index/2),
 * then in fp32 sums[l] += (d_w*d_a) * aux[l] and sumf -= (dmin_w*d_a) * sumi;
 * finally sumf += sums[0..7] in order.
 */
#include "b2q_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline float f16at(const uint8_t* p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return b2q_orc_fp16_to_fp32(h);
}

void b2q_orc_q4k_scale_min(const uint8_t* s, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static inline int q4k_quant(const uint8_t* qs, int p) {
    const int g = p / 64, r = p % 64;
    const uint8_t b = qs[32 * g + (r % 32)];
    return r < 32 ? (b & 15) : (b >> 4);
}

void b2q_orc_dequantize_row_q4_K(const uint8_t* y, float* x, int64_t k) {
    for (int64_t i = 0; i < k / B2Q_ORC_QK_K; ++i) {
        const uint8_t* b = y + i * B2Q_ORC_Q4_K_BYTES;
        const float d = f16at(b), dmin = f16at(b + 2);
        for (int j = 0; j < 8; ++j) {
            int sc, m;
            b2q_orc_q4k_scale_min(b + 4, j, &sc, &m);
            const float d1 = d * (float)sc, m1 = dmin * (float)m;
            for (int l = 0; l < 32; ++l) x[i * 256 + 32 * j + l] = d1 * (float)q4k_quant(b + 16, 32 * j + l) - m1;
        }
    }
}

void b2q_orc_quantize_row_q8_K(const float* x, uint8_t* y, int64_t k) {
    for (int64_t i = 0; i < k / B2Q_ORC_QK_K; ++i) {
        const float* xb = x + i * 256;
        uint8_t* b = y + i * B2Q_ORC_Q8_K_BYTES;
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < 256; ++j) {
            const float ax = fabsf(xb[j]);
            if (ax > amax) {
                amax = ax;
                max = xb[j];
            }
        }
        int8_t* qs = (int8_t*)(b + 4);
        int16_t bs[16];
        if (amax == 0.0f) {
            const float z = 0.0f;
            memcpy(b, &z, 4);
            memset(qs, 0, 256);
            memset(bs, 0, sizeof bs);
        } else {
            const float iscale = -127.0f / max;
            for (int j = 0; j < 256; ++j) {
                const int v = (int)rintf(iscale * xb[j]); /* round half to even (default mode) */
                qs[j] = (int8_t)(v < 127 ? v : 127);
            }
            for (int j = 0; j < 16; ++j) {
                int s = 0;
                for (int l = 0; l < 16; ++l) s += qs[16 * j + l];
                bs[j] = (int16_t)s;
            }
            const float d = 1.0f / iscale;
            memcpy(b, &d, 4);
        }
        memcpy(b + 4 + 256, bs, sizeof bs);
    }
}

float b2q_orc_vec_dot_q4_K_q8_K(const uint8_t* w, const uint8_t* a, int64_t k) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sumf = 0.0f;
    for (int64_t i = 0; i < k / B2Q_ORC_QK_K; ++i) {
        const uint8_t* wb = w + i * B2Q_ORC_Q4_K_BYTES;
        const uint8_t* ab = a + i * B2Q_ORC_Q8_K_BYTES;
        float da;
        memcpy(&da, ab, 4);
        const int8_t* q8 = (const int8_t*)(ab + 4);
        int16_t bs[16];
        memcpy(bs, ab + 4 + 256, sizeof bs);
        int sc[8], mn[8];
        for (int j = 0; j < 8; ++j) b2q_orc_q4k_scale_min(wb + 4, j, &sc[j], &mn[j]);
        int32_t sumi = 0;
        for (int j = 0; j < 16; ++j) sumi += (int32_t)bs[j] * mn[j / 2];
        int32_t aux[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int p = 0; p < 256; ++p) aux[p % 8] += sc[p / 32] * (q4k_quant(wb + 16, p) * (int32_t)q8[p]);
        const float d = f16at(wb) * da;
        for (int l = 0; l < 8; ++l) sums[l] += d * (float)aux[l];
        const float dmin = f16at(wb + 2) * da;
        sumf -= dmin * (float)sumi;
    }
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}

int b2q_orc_mul_mat_q4_K(const uint8_t* w, int64_t w_row_stride, int64_t N, const float* x,
                         int64_t x_row_stride_floats, int64_t M, int64_t K, float* y,
                         int64_t y_row_stride_floats, int nthreads) {
    const int64_t arow = K / B2Q_ORC_QK_K * B2Q_ORC_Q8_K_BYTES;
    uint8_t* a = (uint8_t*)malloc((size_t)(arow * (M > 0 ? M : 1)));
    if (!a) return -1;
    for (int64_t m = 0; m < M; ++m) b2q_orc_quantize_row_q8_K(x + m * x_row_stride_floats, a + m * arow, K);
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            y[m * y_row_stride_floats + n] = b2q_orc_vec_dot_q4_K_q8_K(w + n * w_row_stride, a + m * arow, K);
    (void)nthreads;
    free(a);
    return 0;
}
