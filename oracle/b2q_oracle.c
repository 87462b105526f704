/*
 * b2q_oracle.c -- CPU restatement of ggml's Q8_0 / Q4_0 mul_mat (test
 * infrastructure only; see b2q_oracle.h for the scope and the pins).
 *
 * Compile with -ffp-contract=off: every multiply and add below is a separate
 * IEEE fp32 operation unless fmaf() is written explicitly, exactly as the
 * restated algorithm specifies.
 */
#include "b2q_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ fp16 */

uint16_t b2q_orc_fp32_to_fp16(float f) {
    /* IEEE binary32 -> binary16, round to nearest, ties to even (the rounding
     * of x86 F16C vcvtps2ph with imm 0, which ggml uses for block scales). */
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
    if (ax >= 0x38800000u) {                                  /* normal half */
        uint32_t r = ax - 0x38000000u;                         /* rebias 127 -> 15 */
        r += 0x0fffu + ((r >> 13) & 1u);
        return (uint16_t)(sign | (r >> 13));
    }
    /* subnormal half: value = round(|f| * 2^24) * 2^-24 */
    const uint32_t e = ax >> 23;
    if (e == 0) return (uint16_t)sign; /* fp32 subnormals are far below 2^-25 */
    const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t s = 126u - e; /* >= 14 */
    if (s > 24u) return (uint16_t)sign;
    uint32_t q = m >> s;
    const uint32_t rem = m & ((1u << s) - 1u);
    const uint32_t half = 1u << (s - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

float b2q_orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu;
    const uint32_t m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else { /* subnormal: m * 2^-24, exact in fp32 */
            float v = (float)m * 5.9604644775390625e-08f;
            memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

void b2q_orc_fp32_to_fp16_n(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = b2q_orc_fp32_to_fp16(x[i]);
}

static inline void put_f16(uint8_t* p, uint16_t h) {
    p[0] = (uint8_t)(h & 0xff);
    p[1] = (uint8_t)(h >> 8);
}
static inline uint16_t get_f16(const uint8_t* p) {
    return (uint16_t)(p[0] | ((uint16_t)p[1] << 8));
}

/* ------------------------------------------------------------ quantizers */

static inline float block_amax(const float* x) {
    float amax = 0.0f;
    for (int j = 0; j < B2Q_ORC_QK; ++j) {
        const float v = fabsf(x[j]);
        if (v > amax) amax = v;
    }
    return amax;
}

void b2q_orc_quantize_row_q8_0_ref(const float* x, uint8_t* y, int64_t k) {
    /* ggml scalar reference: d = amax/127; id = 1/d; q = roundf(x*id). */
    const int64_t nb = k / B2Q_ORC_QK;
    for (int64_t b = 0; b < nb; ++b) {
        const float* xb = x + b * B2Q_ORC_QK;
        uint8_t* yb = y + b * B2Q_ORC_Q8_0_BYTES;
        const float amax = block_amax(xb);
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        put_f16(yb, b2q_orc_fp32_to_fp16(d));
        for (int j = 0; j < B2Q_ORC_QK; ++j) {
            const float v = xb[j] * id;
            yb[2 + j] = (uint8_t)(int8_t)roundf(v);
        }
    }
}

static void quantize_row_q8_0_x86(const float* x, uint8_t* y, int64_t k) {
    /* ggml-cpu x86 SIMD from_float: d = amax/127; id = 127/amax;
     * q = round-to-nearest-even(x*id), saturating pack to int8. */
    const int64_t nb = k / B2Q_ORC_QK;
    for (int64_t b = 0; b < nb; ++b) {
        const float* xb = x + b * B2Q_ORC_QK;
        uint8_t* yb = y + b * B2Q_ORC_Q8_0_BYTES;
        const float amax = block_amax(xb);
        const float d = amax / 127.0f;
        const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
        put_f16(yb, b2q_orc_fp32_to_fp16(d));
        for (int j = 0; j < B2Q_ORC_QK; ++j) {
            const float v = nearbyintf(xb[j] * id); /* default mode: ties to even */
            int q = (int)v;
            if (q > 127) q = 127;
            if (q < -128) q = -128;
            yb[2 + j] = (uint8_t)(int8_t)q;
        }
    }
}

void b2q_orc_quantize_row_q8_0_act(const float* x, uint8_t* y, int64_t k, int variant) {
    if (variant == B2Q_ORC_ACT_REF)
        b2q_orc_quantize_row_q8_0_ref(x, y, k);
    else
        quantize_row_q8_0_x86(x, y, k);
}

void b2q_orc_quantize_row_q4_0_ref(const float* x, uint8_t* y, int64_t k) {
    /* ggml reference Q4_0: the signed element of largest magnitude (first on
     * ties) sets d = max/-8; q = min(15, trunc(x*id + 8.5)). */
    const int64_t nb = k / B2Q_ORC_QK;
    for (int64_t b = 0; b < nb; ++b) {
        const float* xb = x + b * B2Q_ORC_QK;
        uint8_t* yb = y + b * B2Q_ORC_Q4_0_BYTES;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < B2Q_ORC_QK; ++j) {
            const float v = xb[j];
            if (amax < fabsf(v)) {
                amax = fabsf(v);
                max = v;
            }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        put_f16(yb, b2q_orc_fp32_to_fp16(d));
        for (int j = 0; j < B2Q_ORC_QK / 2; ++j) {
            const float x0 = xb[j] * id;
            const float x1 = xb[j + 16] * id;
            int q0 = (int)truncf(x0 + 8.5f);
            int q1 = (int)truncf(x1 + 8.5f);
            if (q0 > 15) q0 = 15;
            if (q1 > 15) q1 = 15;
            if (q0 < 0) q0 = 0;
            if (q1 < 0) q1 = 0;
            yb[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void b2q_orc_quantize_rows(int type, const float* x, uint8_t* y, int64_t nrows, int64_t k,
                           int act_variant) {
    const int64_t nb = k / B2Q_ORC_QK;
    for (int64_t r = 0; r < nrows; ++r) {
        if (type == B2Q_ORC_TYPE_Q4_0)
            b2q_orc_quantize_row_q4_0_ref(x + r * k, y + r * nb * B2Q_ORC_Q4_0_BYTES, k);
        else if (act_variant < 0)
            b2q_orc_quantize_row_q8_0_ref(x + r * k, y + r * nb * B2Q_ORC_Q8_0_BYTES, k);
        else
            b2q_orc_quantize_row_q8_0_act(x + r * k, y + r * nb * B2Q_ORC_Q8_0_BYTES, k,
                                          act_variant);
    }
}

static inline int unpack_codes(int wtype, const uint8_t* blk, int8_t q[32]) {
    if (wtype == B2Q_ORC_TYPE_Q4_0) {
        for (int j = 0; j < 16; ++j) {
            q[j] = (int8_t)((blk[2 + j] & 0x0f) - 8);
            q[j + 16] = (int8_t)((blk[2 + j] >> 4) - 8);
        }
        return B2Q_ORC_Q4_0_BYTES;
    }
    for (int j = 0; j < 32; ++j) q[j] = (int8_t)blk[2 + j];
    return B2Q_ORC_Q8_0_BYTES;
}

void b2q_orc_dequantize_row(int type, const uint8_t* y, float* x, int64_t k) {
    const int64_t nb = k / B2Q_ORC_QK;
    const int bytes = type == B2Q_ORC_TYPE_Q4_0 ? B2Q_ORC_Q4_0_BYTES : B2Q_ORC_Q8_0_BYTES;
    for (int64_t b = 0; b < nb; ++b) {
        int8_t q[32];
        const uint8_t* blk = y + b * bytes;
        unpack_codes(type, blk, q);
        const float d = b2q_orc_fp16_to_fp32(get_f16(blk));
        for (int j = 0; j < 32; ++j) x[b * 32 + j] = (float)q[j] * d;
    }
}

/* --------------------------------------------------------------- vec_dot */

float b2q_orc_vec_dot(int wtype, const uint8_t* w, const uint8_t* a, int64_t k) {
    const int64_t nb = k / B2Q_ORC_QK;
    const int wbytes = wtype == B2Q_ORC_TYPE_Q4_0 ? B2Q_ORC_Q4_0_BYTES : B2Q_ORC_Q8_0_BYTES;
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* wb = w + b * wbytes;
        const uint8_t* ab = a + b * B2Q_ORC_Q8_0_BYTES;
        int8_t qw[32];
        unpack_codes(wtype, wb, qw);
        const float d = b2q_orc_fp16_to_fp32(get_f16(wb)) * b2q_orc_fp16_to_fp32(get_f16(ab));
        for (int l = 0; l < 8; ++l) {
            int32_t s = 0;
            for (int i = 4 * l; i < 4 * l + 4; ++i) s += (int32_t)qw[i] * (int32_t)(int8_t)ab[2 + i];
            lane[l] = fmaf(d, (float)s, lane[l]);
        }
    }
    const float r0 = lane[4] + lane[0], r1 = lane[5] + lane[1];
    const float r2 = lane[6] + lane[2], r3 = lane[7] + lane[3];
    return (r0 + r2) + (r1 + r3);
}

void b2q_orc_block_dots(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                        const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                        int32_t* dots) {
    const int64_t nb = K / B2Q_ORC_QK;
    const int wbytes = wtype == B2Q_ORC_TYPE_Q4_0 ? B2Q_ORC_Q4_0_BYTES : B2Q_ORC_Q8_0_BYTES;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            for (int64_t b = 0; b < nb; ++b) {
                int8_t qw[32];
                unpack_codes(wtype, w + n * w_row_stride + b * wbytes, qw);
                const uint8_t* ab = a + m * a_row_stride + b * B2Q_ORC_Q8_0_BYTES;
                int32_t s = 0;
                for (int i = 0; i < 32; ++i) s += (int32_t)qw[i] * (int32_t)(int8_t)ab[2 + i];
                dots[(m * N + n) * nb + b] = s;
            }
}

void b2q_orc_mul_mat_q(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                       const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                       float* y, int64_t y_row_stride_floats, int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t m = 0; m < M; ++m)
        for (int64_t n = 0; n < N; ++n)
            y[m * y_row_stride_floats + n] =
                b2q_orc_vec_dot(wtype, w + n * w_row_stride, a + m * a_row_stride, K);
    (void)nthreads;
}

int b2q_orc_mul_mat(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                    const float* x, int64_t x_row_stride_floats, int64_t M, int64_t K,
                    int act_variant, float* y, int64_t y_row_stride_floats, int nthreads) {
    const int64_t arow = K / B2Q_ORC_QK * B2Q_ORC_Q8_0_BYTES;
    uint8_t* a = (uint8_t*)malloc((size_t)(arow * (M > 0 ? M : 1)));
    if (!a) return -1;
    for (int64_t m = 0; m < M; ++m)
        b2q_orc_quantize_row_q8_0_act(x + m * x_row_stride_floats, a + m * arow, K, act_variant);
    b2q_orc_mul_mat_q(wtype, w, w_row_stride, N, a, arow, M, K, y, y_row_stride_floats, nthreads);
    free(a);
    return 0;
}

void b2q_orc_mul_mat_f64(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                         const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                         double* y) {
    float* wr = (float*)malloc(sizeof(float) * (size_t)K);
    float* ar = (float*)malloc(sizeof(float) * (size_t)K);
    for (int64_t m = 0; m < M; ++m) {
        b2q_orc_dequantize_row(B2Q_ORC_TYPE_Q8_0, a + m * a_row_stride, ar, K);
        for (int64_t n = 0; n < N; ++n) {
            b2q_orc_dequantize_row(wtype, w + n * w_row_stride, wr, K);
            double s = 0.0;
            for (int64_t i = 0; i < K; ++i) s += (double)wr[i] * (double)ar[i];
            y[m * N + n] = s;
        }
    }
    free(wr);
    free(ar);
}

/* ------------------------------------------------------------ generators */

void b2q_orc_philox4x32_10(uint64_t seed, uint64_t counter, uint32_t out[4]) {
    /* Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, SC'11). */
    uint32_t c0 = (uint32_t)counter, c1 = (uint32_t)(counter >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n1 = (uint32_t)p1;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        const uint32_t n3 = (uint32_t)p0;
        c0 = n0;
        c1 = n1;
        c2 = n2;
        c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

void b2q_orc_fill_normal(float* x, int64_t n, uint64_t seed, float mean, float std) {
    /* Box-Muller: each Philox call yields 4 words -> 2 uniform pairs -> 4 normals. */
    for (int64_t i = 0; i < n; i += 4) {
        uint32_t r[4];
        b2q_orc_philox4x32_10(seed, (uint64_t)(i / 4), r);
        for (int p = 0; p < 2; ++p) {
            const double u1 = ((double)r[2 * p] + 1.0) / 4294967296.0; /* (0,1] */
            const double u2 = (double)r[2 * p + 1] / 4294967296.0;     /* [0,1) */
            const double rad = sqrt(-2.0 * log(u1));
            const double th = 6.283185307179586 * u2;
            const double z0 = rad * cos(th), z1 = rad * sin(th);
            if (i + 2 * p < n) x[i + 2 * p] = (float)(mean + std * z0);
            if (i + 2 * p + 1 < n) x[i + 2 * p + 1] = (float)(mean + std * z1);
        }
    }
}

/* ------------------------------------------------------------------ GELU */

/* ggml-cpu/vec.h (v0.21.0): GELU_COEF_A, SQRT_2_OVER_PI and ggml_gelu_f32,
 * tabulated over fp16 inputs (GGML_GELU_FP16).  See b2q_oracle.h. */
static float gelu_f32(float f, int contract) {
  const float kA = 0.044715f;
  const float kS = 0.79788456080286535587989211986876f;
  const float inner = contract ? fmaf(kA * f, f, 1.0f) : 1.0f + (kA * f) * f;
  return (0.5f * f) * (1.0f + tanhf((kS * f) * inner));
}

void b2q_orc_gelu_table(uint16_t* table, int contract) {
  for (uint32_t h = 0; h < 65536u; ++h)
    table[h] = b2q_orc_fp32_to_fp16(gelu_f32(b2q_orc_fp16_to_fp32((uint16_t)h), contract));
}

float b2q_orc_gelu(float x, int contract) {
  if (x <= -10.0f) return 0.0f;
  if (x >= 10.0f) return x;
  const float f = b2q_orc_fp16_to_fp32(b2q_orc_fp32_to_fp16(x));
  return b2q_orc_fp16_to_fp32(b2q_orc_fp32_to_fp16(gelu_f32(f, contract)));
}

void b2q_orc_gelu_n(const float* x, float* y, int64_t n, int contract) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) y[i] = b2q_orc_gelu(x[i], contract);
}

/* ---------------------------------------------------------- LayerNorm */

void b2q_orc_norm_modulate(const float* x, int64_t m, int64_t c, int64_t ldx_floats, float eps,
                           const float* scale, const float* shift, float* y, int64_t ldy_floats) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < m; ++r) {
    const float* xr = x + r * ldx_floats;
    float* yr = y + r * ldy_floats;
    double sum = 0.0;
    for (int64_t i = 0; i < c; ++i) sum += (double)xr[i];
    const float mean = (float)sum / (float)c;
    double sum2 = 0.0;
    for (int64_t i = 0; i < c; ++i) {
      const float v = xr[i] - mean;
      yr[i] = v;
      sum2 += (double)(v * v);
    }
    const float var = (float)(sum2 / (double)c);
    const float rs = 1.0f / sqrtf(var + eps);
    for (int64_t i = 0; i < c; ++i) {
      float h = yr[i] * rs;
      if (scale) h = h * scale[i] + h;
      if (shift) h = h + shift[i];
      yr[i] = h;
    }
  }
}

int b2q_orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
