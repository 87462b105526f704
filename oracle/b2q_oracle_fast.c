/*
 * b2q_oracle_fast.c -- vectorised, multi-threaded form of the oracle's
 * mul_mat with the SAME arithmetic as b2q_orc_vec_dot (test infrastructure:
 * the timed CPU baseline of bench.py; tests check it bit-for-bit against the
 * scalar oracle).
 *
 * Lane structure of one block (32 products): 8 int32 lanes, lane l = products
 * 4l..4l+3, converted to fp32 and accumulated with one fused multiply-add per
 * block by the block's scale product; the 8 lanes are reduced pairwise at the
 * end in a fixed order.  On AVX2 the int8 x int8 products use the unsigned x
 * signed byte multiply-add with the sign moved onto the second operand
 * (|w| * sign(a, w)), which yields the same exact 4-product partials.
 */
#include "b2q_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static float g_f16_table[65536];
static int g_f16_table_ready = 0;

static void init_f16_table(void) {
    if (g_f16_table_ready) return;
#ifdef _OPENMP
#pragma omp critical(b2q_f16_table)
#endif
    {
        if (!g_f16_table_ready) {
            for (uint32_t h = 0; h < 65536u; ++h) g_f16_table[h] = b2q_orc_fp16_to_fp32((uint16_t)h);
            g_f16_table_ready = 1;
        }
    }
}

static inline float f16at(const uint8_t* p) {
    return g_f16_table[(uint16_t)(p[0] | ((uint16_t)p[1] << 8))];
}

#define ROWS 4

static inline float hsum8_fixed(const float l[8]) {
    const float r0 = l[4] + l[0], r1 = l[5] + l[1], r2 = l[6] + l[2], r3 = l[7] + l[3];
    return (r0 + r2) + (r1 + r3);
}

__attribute__((target("avx2,fma"))) static inline __m256i load_wcodes_avx2(int wtype,
                                                                          const uint8_t* wb) {
    if (wtype == B2Q_ORC_TYPE_Q4_0) {
        const __m128i packed = _mm_loadu_si128((const __m128i*)(wb + 2));
        const __m128i lo = _mm_and_si128(packed, _mm_set1_epi8(0x0f));
        const __m128i hi = _mm_and_si128(_mm_srli_epi16(packed, 4), _mm_set1_epi8(0x0f));
        const __m256i q = _mm256_set_m128i(hi, lo);
        return _mm256_sub_epi8(q, _mm256_set1_epi8(8));
    }
    return _mm256_loadu_si256((const __m256i*)(wb + 2));
}

/* One weight row against up to ROWS activation rows, AVX2 (maddubs path). */
__attribute__((target("avx2,fma"))) static void dot_avx2(int wtype, const uint8_t* w,
                                                         const uint8_t* const* a, int na,
                                                         int64_t nb, float* out) {
    const int wbytes = wtype == B2Q_ORC_TYPE_Q4_0 ? B2Q_ORC_Q4_0_BYTES : B2Q_ORC_Q8_0_BYTES;
    __m256 acc[ROWS];
    for (int r = 0; r < ROWS; ++r) acc[r] = _mm256_setzero_ps();
    const __m256i ones = _mm256_set1_epi16(1);
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* wb = w + b * wbytes;
        const __m256i qw = load_wcodes_avx2(wtype, wb);
        const __m256i ax = _mm256_sign_epi8(qw, qw);
        const float dw = f16at(wb);
        for (int r = 0; r < na; ++r) {
            const uint8_t* ab = a[r] + b * B2Q_ORC_Q8_0_BYTES;
            const __m256i qa = _mm256_loadu_si256((const __m256i*)(ab + 2));
            const __m256i sy = _mm256_sign_epi8(qa, qw);
            const __m256i p32 = _mm256_madd_epi16(_mm256_maddubs_epi16(ax, sy), ones);
            const __m256 d = _mm256_set1_ps(dw * f16at(ab));
            acc[r] = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(p32), acc[r]);
        }
    }
    for (int r = 0; r < na; ++r) {
        float l[8];
        _mm256_storeu_ps(l, acc[r]);
        out[r] = hsum8_fixed(l);
    }
}

/* Same with the AVX-512 VNNI byte dot (vpdpbusd on 256-bit vectors). */
__attribute__((target("avx2,fma,avx512f,avx512vl,avx512vnni"))) static void dot_vnni(
    int wtype, const uint8_t* w, const uint8_t* const* a, int na, int64_t nb, float* out) {
    const int wbytes = wtype == B2Q_ORC_TYPE_Q4_0 ? B2Q_ORC_Q4_0_BYTES : B2Q_ORC_Q8_0_BYTES;
    __m256 acc[ROWS];
    for (int r = 0; r < ROWS; ++r) acc[r] = _mm256_setzero_ps();
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* wb = w + b * wbytes;
        __m256i qw;
        if (wtype == B2Q_ORC_TYPE_Q4_0) {
            const __m128i packed = _mm_loadu_si128((const __m128i*)(wb + 2));
            const __m128i lo = _mm_and_si128(packed, _mm_set1_epi8(0x0f));
            const __m128i hi = _mm_and_si128(_mm_srli_epi16(packed, 4), _mm_set1_epi8(0x0f));
            qw = _mm256_sub_epi8(_mm256_set_m128i(hi, lo), _mm256_set1_epi8(8));
        } else {
            qw = _mm256_loadu_si256((const __m256i*)(wb + 2));
        }
        const __m256i ax = _mm256_sign_epi8(qw, qw);
        const float dw = f16at(wb);
        for (int r = 0; r < na; ++r) {
            const uint8_t* ab = a[r] + b * B2Q_ORC_Q8_0_BYTES;
            const __m256i qa = _mm256_loadu_si256((const __m256i*)(ab + 2));
            const __m256i sy = _mm256_sign_epi8(qa, qw);
            const __m256i p32 = _mm256_dpbusd_epi32(_mm256_setzero_si256(), ax, sy);
            const __m256 d = _mm256_set1_ps(dw * f16at(ab));
            acc[r] = _mm256_fmadd_ps(d, _mm256_cvtepi32_ps(p32), acc[r]);
        }
    }
    for (int r = 0; r < na; ++r) {
        float l[8];
        _mm256_storeu_ps(l, acc[r]);
        out[r] = hsum8_fixed(l);
    }
}

static void dot_scalar(int wtype, const uint8_t* w, const uint8_t* const* a, int na, int64_t nb,
                       float* out) {
    for (int r = 0; r < na; ++r) out[r] = b2q_orc_vec_dot(wtype, w, a[r], nb * B2Q_ORC_QK);
}

typedef void (*dot_fn)(int, const uint8_t*, const uint8_t* const*, int, int64_t, float*);

static dot_fn pick_dot(const char** isa) {
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl") &&
        __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) {
        if (isa) *isa = "avx512vnni";
        return dot_vnni;
    }
    if (__builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma")) {
        if (isa) *isa = "avx2";
        return dot_avx2;
    }
    if (isa) *isa = "scalar";
    return dot_scalar;
}

const char* b2q_orc_isa(void) {
    const char* isa = "scalar";
    pick_dot(&isa);
    return isa;
}

int b2q_orc_mul_mat_q_fast(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                           const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                           float* y, int64_t y_row_stride_floats, int nthreads) {
    init_f16_table();
    const dot_fn dot = pick_dot(NULL);
    const int64_t nb = K / B2Q_ORC_QK;
    const int64_t mgroups = (M + ROWS - 1) / ROWS;
    const int64_t NCH = 64; /* weight rows per task: keeps a weight panel in L2 */
    const int64_t nchunks = (N + NCH - 1) / NCH;
    const int64_t ntasks = mgroups * nchunks;
    int used = 1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    used = nthreads;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
#endif
    for (int64_t t = 0; t < ntasks; ++t) {
        const int64_t nc = t / mgroups, mg = t % mgroups;
        const int64_t m0 = mg * ROWS;
        const int na = (int)((M - m0) < ROWS ? (M - m0) : ROWS);
        const uint8_t* arows[ROWS];
        for (int r = 0; r < na; ++r) arows[r] = a + (m0 + r) * a_row_stride;
        const int64_t n1 = (nc + 1) * NCH < N ? (nc + 1) * NCH : N;
        for (int64_t n = nc * NCH; n < n1; ++n) {
            float out[ROWS];
            dot(wtype, w + n * w_row_stride, arows, na, nb, out);
            for (int r = 0; r < na; ++r) y[(m0 + r) * y_row_stride_floats + n] = out[r];
        }
    }
    (void)nthreads;
    return used;
}

int b2q_orc_mul_mat_fast(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                         const float* x, int64_t x_row_stride_floats, int64_t M, int64_t K,
                         int act_variant, float* y, int64_t y_row_stride_floats, int nthreads) {
    const int64_t arow = K / B2Q_ORC_QK * B2Q_ORC_Q8_0_BYTES;
    uint8_t* a = (uint8_t*)malloc((size_t)(arow * (M > 0 ? M : 1)));
    if (!a) return -1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int64_t m = 0; m < M; ++m)
        b2q_orc_quantize_row_q8_0_act(x + m * x_row_stride_floats, a + m * arow, K, act_variant);
    const int used =
        b2q_orc_mul_mat_q_fast(wtype, w, w_row_stride, N, a, arow, M, K, y, y_row_stride_floats,
                               nthreads);
    free(a);
    return used;
}
