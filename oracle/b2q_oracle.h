/*
 * b2q_oracle.h -- CPU restatement of ggml's Q8_0 / Q4_0 quantized mul_mat.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker the CUDA path is compared
 * against (tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg).
 * Nothing in the product library links, loads or calls it.
 *
 * What it restates (ggml v0.21.0, the pinned submodule of the reference,
 * cpp_ggml/CMakeLists.txt:126; the submodule is empty in the reference
 * checkout, so the semantics are restated from the published block formats
 * and pinned against gguf-py 0.19.0's bit-exact ggml quantizers):
 *
 *   block_q8_0 = { fp16 d; int8 qs[32]; }                       34 bytes
 *   block_q4_0 = { fp16 d; uint8 qs[16]; }  element j -> low nibble of qs[j],
 *                element j+16 -> high nibble of qs[j], value = nibble - 8     18 bytes
 *
 *   GGML_OP_MUL_MAT(src0 = W [K,N] Q8_0|Q4_0, src1 = X [K,M] F32) -> Y [N,M] F32
 *     1. every src1 row is converted to Q8_0 by the CPU backend's from_float
 *        (the activation quantizer; both weight types use Q8_0 activations);
 *     2. Y[m][n] = vec_dot(W row n, Xq row m)
 *              = sum_b fp32(dw[n,b]) * fp32(da[m,b]) * S_b,   S_b = sum_{i<32} qw*qa  (int32)
 *   Call sites in the reference: cpp_ggml/src/graph_builder.cpp:44-60 (gb_linear),
 *   cpp_ggml/src/ss_flow_graph.cpp:85-112, cpp_ggml/src/matmul_backend_test.cpp:36-37.
 *
 * Two activation-quantizer variants exist in ggml and both are restated:
 *   B2Q_ORC_ACT_X86 : the x86 SIMD from_float the CPU backend runs on the
 *                     x86 host:  d = amax/127, inverse = 127/amax, round to
 *                     nearest-even.  (Recalled upstream semantics: no copy
 *                     of that source exists on this machine -> unpinned.)
 *   B2Q_ORC_ACT_REF : the scalar reference quantizer (also used for weights by
 *                     ggml_quantize_chunk, matmul_backend_test.cpp:49):
 *                     d = amax/127, inverse = 1/d, round half away from zero.
 *                     Pinned byte-for-byte against gguf-py's Q8_0 quantizer.
 *
 * The fp32 dot follows the x86 AVX2 accumulation order: 8 fp32 lanes, lane l
 * holding the int32 partial of products 4l..4l+3 of each block, accumulated
 * with one fused multiply-add per block, then a fixed pairwise lane reduction.
 */
#ifndef B2Q_ORACLE_H
#define B2Q_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { B2Q_ORC_QK = 32, B2Q_ORC_Q8_0_BYTES = 34, B2Q_ORC_Q4_0_BYTES = 18 };
/* ggml type ids (ggml.h enum ggml_type numbering) */
enum { B2Q_ORC_TYPE_F32 = 0, B2Q_ORC_TYPE_Q4_0 = 2, B2Q_ORC_TYPE_Q8_0 = 8 };
enum { B2Q_ORC_ACT_X86 = 0, B2Q_ORC_ACT_REF = 1 };

uint16_t b2q_orc_fp32_to_fp16(float f);
float b2q_orc_fp16_to_fp32(uint16_t h);
void b2q_orc_fp32_to_fp16_n(const float* x, uint16_t* y, int64_t n);

/* Weight quantizers (ggml reference semantics). k must be a multiple of 32. */
void b2q_orc_quantize_row_q8_0_ref(const float* x, uint8_t* y, int64_t k);
void b2q_orc_quantize_row_q4_0_ref(const float* x, uint8_t* y, int64_t k);
/* Activation quantizer, variant B2Q_ORC_ACT_X86 or B2Q_ORC_ACT_REF. */
void b2q_orc_quantize_row_q8_0_act(const float* x, uint8_t* y, int64_t k, int variant);
/* Row-wise helpers: nrows rows of k values, src row stride k floats, dst row
 * stride k/32 blocks. */
void b2q_orc_quantize_rows(int type, const float* x, uint8_t* y, int64_t nrows, int64_t k,
                           int act_variant);
void b2q_orc_dequantize_row(int type, const uint8_t* y, float* x, int64_t k);

/* One vec_dot, x86 lane order.  w: one weight row (Q8_0 or Q4_0), a: one
 * Q8_0 activation row, k elements. */
float b2q_orc_vec_dot(int wtype, const uint8_t* w, const uint8_t* a, int64_t k);

/* Per-block int32 dot products: dots[(m*N + n)*KB + b] = S_b(n, m). */
void b2q_orc_block_dots(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                        const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                        int32_t* dots);

/* Full mul_mat on pre-quantized activations (a: M rows of Q8_0 blocks). */
void b2q_orc_mul_mat_q(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                       const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                       float* y, int64_t y_row_stride_floats, int nthreads);
/* Full mul_mat from fp32 activations (quantize + dot), as GGML_OP_MUL_MAT runs.
 * x: M rows, row stride x_row_stride_floats.  Scratch for the quantized rows
 * is allocated internally. Returns 0 on success. */
int b2q_orc_mul_mat(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                    const float* x, int64_t x_row_stride_floats, int64_t M, int64_t K,
                    int act_variant, float* y, int64_t y_row_stride_floats, int nthreads);

/* Vectorised (AVX2 / AVX-512 VNNI when the host has it) + OpenMP variant of
 * b2q_orc_mul_mat_q with identical arithmetic; used as the timed CPU baseline.
 * Returns the number of threads used. */
int b2q_orc_mul_mat_q_fast(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                           const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                           float* y, int64_t y_row_stride_floats, int nthreads);
/* Same, starting from fp32 activations (parallel activation quantize). */
int b2q_orc_mul_mat_fast(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                         const float* x, int64_t x_row_stride_floats, int64_t M, int64_t K,
                         int act_variant, float* y, int64_t y_row_stride_floats, int nthreads);

/* fp64 reference of the dequantized product (second, order-free check). */
void b2q_orc_mul_mat_f64(int wtype, const uint8_t* w, int64_t w_row_stride, int64_t N,
                         const uint8_t* a, int64_t a_row_stride, int64_t M, int64_t K,
                         double* y);

/* Counter-based generator shared with the device (Philox4x32-10, Salmon et
 * al., SC'11): element i of stream (seed) -> 4 uint32 words. */
void b2q_orc_philox4x32_10(uint64_t seed, uint64_t counter, uint32_t out[4]);
/* Normal(mean, std) fp32 values via Box-Muller on Philox words. */
void b2q_orc_fill_normal(float* x, int64_t n, uint64_t seed, float mean, float std);

/* ---- Q4_K weights x Q8_K activations (b2q_oracle_k.c; layouts there) ---- */
#define B2Q_ORC_TYPE_Q4_K 12
#define B2Q_ORC_QK_K 256
#define B2Q_ORC_Q4_K_BYTES 144
#define B2Q_ORC_Q8_K_BYTES 292
void b2q_orc_q4k_scale_min(const uint8_t* scales12, int j, int* sc, int* m);
void b2q_orc_dequantize_row_q4_K(const uint8_t* y, float* x, int64_t k);
void b2q_orc_quantize_row_q8_K(const float* x, uint8_t* y, int64_t k);
float b2q_orc_vec_dot_q4_K_q8_K(const uint8_t* w, const uint8_t* a, int64_t k);
/* Full mul_mat from fp32 activations (Q8_K quantize + dot).  Returns 0. */
int b2q_orc_mul_mat_q4_K(const uint8_t* w, int64_t w_row_stride, int64_t N, const float* x,
                         int64_t x_row_stride_floats, int64_t M, int64_t K, float* y,
                         int64_t y_row_stride_floats, int nthreads);

/* ggml_gelu on the CPU backend (ggml v0.21.0 ggml-cpu/vec.h, the
 * GGML_GELU_FP16 build, which is the default): outside (-10, 10) the result is
 * 0 (x <= -10) or x (x >= 10); inside, x is rounded to fp16 and looked up in a
 * 65536-entry table whose entry h is
 *   fp16( 0.5f*f*(1.0f + tanhf(SQRT_2_OVER_PI*f*(1.0f + GELU_COEF_A*f*f))) ),
 * f = fp32(h), evaluated left to right, one IEEE op per step.  contract != 0
 * evaluates 1 + GELU_COEF_A*f*f as one fmaf, as a compiler that contracts
 * (-ffp-contract=fast with FMA enabled) builds the table. */
float b2q_orc_gelu(float x, int contract);
void b2q_orc_gelu_n(const float* x, float* y, int64_t n, int contract);
/* The 65536-entry table itself (fp16 bits), for exhaustive comparisons. */
void b2q_orc_gelu_table(uint16_t* table, int contract);

/* ggml_norm (LayerNorm without affine) then the adaLN modulate of the SS-flow
 * blocks, per row of c values (cpp_ggml/src/ss_flow_graph.cpp:45-53,
 * graph_builder.cpp:62-68; ggml v0.21.0 ggml-cpu ops.cpp norm_f32):
 *   sum = Σx (double, sequential) cast to float; mean = sum / c (float);
 *   v = x - mean; var = (Σ (v*v as float), double) / c, cast to float;
 *   h = v * (1 / sqrtf(var + eps)); h = (h*scale + h) if scale; h = h + shift if shift.
 * scale / shift are per column, either may be NULL. */
void b2q_orc_norm_modulate(const float* x, int64_t m, int64_t c, int64_t ldx_floats, float eps,
                           const float* scale, const float* shift, float* y, int64_t ldy_floats);

int b2q_orc_num_threads(void);
const char* b2q_orc_isa(void);

#ifdef __cplusplus
}
#endif

#endif
