/*
 * b2q.h -- C ABI of the B200 (sm_100a) quantized mul_mat library (libb2q).
 *
 * The library replaces, for one operator, the arithmetic that ggml runs when a
 * cpp_ggml graph evaluates GGML_OP_MUL_MAT with GGUF block-quantized weights:
 *
 *     y = ggml_mul_mat(ctx, w, x)      w: ne=[K,N] Q8_0 | Q4_0   (row n contiguous over K)
 *                                      x: ne=[K,M] F32           (row m contiguous over K)
 *                                      y: ne=[N,M] F32, y[m*N + n] = sum_k w[n,k] x[m,k]
 *
 * reached from gb_linear (cpp_ggml/src/graph_builder.cpp:44-60) at every SS
 * flow linear (cpp_ggml/src/ss_flow_graph.cpp:85-112) and SLat flow linear
 * (cpp_ggml/src/slat_flow_graph.cpp:29-40), and exercised directly by
 * cpp_ggml/src/matmul_backend_test.cpp:36-37.  Semantics are those of the ggml
 * CPU backend: every x row is quantized to Q8_0 (32 int8 + fp16 scale per
 * block), then y[m][n] = sum_b fp32(dw[n,b]) * fp32(da[m,b]) * S_b with the
 * int32 block dot S_b = sum_{i<32} qw * qa  (Q4_0: qw = nibble - 8).
 *
 * Conventions
 *   - All data pointers are DEVICE pointers owned by the caller.  `stream` is a
 *     cudaStream_t (NULL = legacy default stream).  Compute calls are
 *     asynchronous, allocate nothing and never synchronise.
 *   - Row strides are in BYTES, like ggml's nb[1]; a weight may be a row-offset
 *     view of a larger tensor (cpp_ggml/src/ss_flow_graph.cpp:38-44).
 *   - Every call returns a b2q_status; nothing aborts, nothing traps on device.
 *     Device-side waits are bounded; a wait that gives up records a code that
 *     b2q_device_status() returns.
 *   - Type ids use ggml's enum ggml_type numbering so a ggml backend can pass
 *     tensor->type straight through.
 */
#ifndef B2Q_H
#define B2Q_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B2Q_API __attribute__((visibility("default")))
#else
#define B2Q_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum b2q_type { B2Q_TYPE_F32 = 0, B2Q_TYPE_F16 = 1, B2Q_TYPE_Q4_0 = 2, B2Q_TYPE_Q8_0 = 8, B2Q_TYPE_Q4_K = 12 };

/* Activation-quantizer variant (fp32 -> Q8_0 rounding).
 *   B2Q_ACT_X86: the from_float of ggml's CPU backend on x86 (the host the
 *                reference runs on): inverse scale 127/amax, ties to even.
 *   B2Q_ACT_REF: ggml's scalar reference quantizer: inverse 1/d, ties away
 *                from zero.
 *   B2Q_ACT_Q8_K: fp32 -> Q8_K (256-value blocks, fp32 scale), the activation
 *                format ggml's CPU backend uses against Q4_K weights; the only
 *                variant Q4_K weights accept, and accepted only with them.
 *
 * Q4_K weights (ggml's shipped 4-bit k-quant, cpp_ggml/models/MODEL_CARD.md:54-74)
 * need K % 256 == 0 and have their own packed layout (three int8 planes and
 * the super-block scales) and prepared-activation layout (Q8_K codes and one
 * fp32 scale per 256 values); size them with the typed functions below.  The
 * untyped size functions and prepared entries serve Q8_0 / Q4_0. */
enum b2q_act_variant { B2Q_ACT_X86 = 0, B2Q_ACT_REF = 1, B2Q_ACT_Q8_K = 2 };

/* Typed sizes (0 when the arguments are not valid for the type):
 * the packed weight, the prepared activations of an activation variant, and
 * the workspace of b2q_mul_mat (packed_weight = 0) / b2q_mul_mat_packed (1). */
B2Q_API size_t b2q_weight_packed_bytes(int wtype, int64_t n, int64_t k);
B2Q_API size_t b2q_act_prepared_bytes(int variant, int64_t m, int64_t k);
B2Q_API size_t b2q_mul_mat_workspace_bytes(int wtype, int64_t m, int64_t n, int64_t k, int packed_weight);

enum b2q_status {
    B2Q_OK = 0,
    B2Q_ERR_INVALID_ARG = 1,  /* null pointer, negative/zero size, K % 32 != 0, ... */
    B2Q_ERR_UNSUPPORTED = 2,  /* type combination or device not supported (needs sm_100) */
    B2Q_ERR_MISALIGNED = 3,   /* pointer or stride violates the stated alignment */
    B2Q_ERR_WORKSPACE = 4,    /* workspace / packed buffer too small */
    B2Q_ERR_CUDA = 5,         /* a CUDA runtime call failed (launch, attribute, ...) */
    B2Q_ERR_DEVICE = 6,       /* a kernel reported a device-side error (bounded wait gave up) */
    B2Q_ERR_TOO_LARGE = 7     /* size beyond what the entry point supports */
};

B2Q_API const char* b2q_status_string(int status);
B2Q_API const char* b2q_version(void);

/* ------------------------------------------------------------ quantize
 * fp32 rows -> ggml block_q8_0 rows (34 bytes per 32 values).
 * Replaces the CPU backend's from_float for GGML_TYPE_Q8_0, which ggml's CPU
 * mul_mat applies to every src1 row before the dot products (the conversion
 * noted at cpp_ggml/src/matmul_backend_test.cpp:171-174).
 * x: nrows rows of k floats (x_row_stride_bytes apart, multiple of 4);
 * y: nrows rows of k/32 blocks (y_row_stride_bytes apart, even).  k % 32 == 0. */
B2Q_API int b2q_quantize_q8_0(const float* x, int64_t nrows, int64_t k, int64_t x_row_stride_bytes,
                      void* y, int64_t y_row_stride_bytes, int variant, void* stream);

/* --------------------------------------------------------- weight packing
 * One-time re-layout of a GGUF weight (Q8_0 or Q4_0 blocks, as loaded by
 * cpp_ggml/src/gguf_loader.cpp:113-133) into the GEMM's layout: int8 codes
 * [n][k] (Q4_0 nibbles widened to code-8) and fp32 scales [k/32][ldn].
 * This is what a ggml buffer type's set_tensor hook runs on upload; the
 * packed buffer then serves every later mul_mat with that weight. */
B2Q_API size_t b2q_weight_packed_size(int64_t n, int64_t k);
B2Q_API int b2q_weight_pack(int wtype, const void* w, int64_t n, int64_t k, int64_t w_row_stride_bytes,
                    void* packed, size_t packed_bytes, void* stream);

/* The same re-layout straight from host memory: the weight rows (raw GGUF
 * blocks, w_row_stride_bytes apart, pageable or pinned) go to the device in
 * chunks through the caller's staging buffer and are packed there, so the raw
 * blocks never need a device allocation of their own.  This is the upload a
 * ggml buffer type runs in set_tensor (ggml_backend_tensor_set from the GGUF
 * loader, cpp_ggml/src/gguf_loader.cpp:133).  staging_bytes must hold at least
 * one row of blocks (k/32 * 34 or 18 bytes); larger staging means fewer
 * chunks.  Asynchronous on `stream`; host_w must stay valid until it is done. */
B2Q_API int b2q_weight_upload(int wtype, const void* host_w, int64_t n, int64_t k, int64_t w_row_stride_bytes,
                              void* staging, size_t staging_bytes, void* packed, size_t packed_bytes,
                              void* stream);

/* --------------------------------------------------------------- mul_mat
 * Scratch needed by b2q_mul_mat (packed_weight = 0) or b2q_mul_mat_packed
 * (packed_weight = 1): the Q8_0 activations in the GEMM's layout, plus the
 * packed weight when it is packed per call. */
B2Q_API size_t b2q_mul_mat_workspace_size(int64_t m, int64_t n, int64_t k, int packed_weight);

/* GGML_OP_MUL_MAT, src0 = w (Q8_0 | Q4_0 blocks), src1 = x (F32), dst = y (F32):
 *   y[m][n] = sum_k w[n][k] x[m][k]  (+ bias[n] if bias != NULL: the
 *   GGML_OP_ADD that gb_linear appends, graph_builder.cpp:58, fused).
 * Replaces ggml's mul_mat for this type combination on the CPU backend and the
 * CUDA backend's ggml_cuda_mul_mat dispatch for it (ggml patch
 * 0001-sam3d-ggml-combined.patch:806-817 routes it to cuBLAS today).
 * Runs: activation quantize (variant) -> weight pack into workspace ->
 * tcgen05 int8 block GEMM with the per-block scale epilogue.
 * Alignment: x rows 16-byte aligned for the vector path (any multiple of 4
 * works), y 4-byte aligned, workspace 256-byte aligned. */
B2Q_API int b2q_mul_mat(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n, int64_t k,
                const float* x, int64_t m, int64_t x_row_stride_bytes, const float* bias,
                float* y, int64_t y_row_stride_bytes, int variant, void* workspace,
                size_t workspace_bytes, void* stream);
/* With wtype = B2Q_TYPE_F16 (src0 F16, ggml_mul_mat's path for F16 GGUF
 * tensors): x is rounded to fp16 (ggml's vec_dot_type for F16, round to nearest
 * even) into the workspace, then a tcgen05 kind::f16 GEMM with fp32
 * accumulation reads the weight rows in place.  k % 8 == 0; w and its row
 * stride 16-byte aligned; variant must be B2Q_ACT_X86 or B2Q_ACT_REF and is
 * not used; workspace = b2q_mul_mat_workspace_bytes(B2Q_TYPE_F16, m, n, k, 0). */

/* Same with a weight packed once by b2q_weight_pack (the production path). */
B2Q_API int b2q_mul_mat_packed(const void* packed, int64_t n, int64_t k, const float* x, int64_t m,
                       int64_t x_row_stride_bytes, const float* bias, float* y,
                       int64_t y_row_stride_bytes, int variant, void* workspace,
                       size_t workspace_bytes, void* stream);

/* ------------------------------------------------------- no-allocation form
 * b2q_mul_mat_packed for callers that may not allocate device memory and have
 * no workspace to lend: code that runs after its memory plan is fixed (a ggml
 * backend computing a graph whose buffers the graph allocator has already
 * placed), or a serving loop that must not call cudaMalloc/cudaFree, which can
 * synchronise the device.  No counterpart exists in the reference: ggml's CPU
 * mul_mat takes its quantized-activation scratch from the work buffer that
 * ggml_graph_plan sizes and the caller provides.
 * The activations go to one fixed device array of B2Q_NOALLOC_SCRATCH_BYTES
 * (32 MiB per device, reserved no later than the first call on each device and
 * held until the process exits), so b2q_act_prepared_bytes(variant, m, k) must
 * not exceed it (Q8_0 activations: about 29.8 M values, e.g. m = 4096 rows up to
 * k = 7168); larger sizes return B2Q_ERR_TOO_LARGE.  The first call on each
 * device sets up (looks up the array's address, with that device current), and
 * so does the first call after the device's CUDA context was replaced (after
 * cudaDeviceReset); make those calls before any stream capture begins.  Every
 * call on a device shares the array, which keeps the last call's contents:
 * calls that can overlap on one device (several streams or threads) race, so
 * serialise them.  Arguments, alignment and results are those of
 * b2q_mul_mat_packed, with the same checks (an unknown variant is
 * B2Q_ERR_INVALID_ARG whatever the size). */
#define B2Q_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
B2Q_API int b2q_mul_mat_packed_noalloc(const void* packed, int64_t n, int64_t k, const float* x,
                                       int64_t m, int64_t x_row_stride_bytes, const float* bias,
                                       float* y, int64_t y_row_stride_bytes, int variant,
                                       void* stream);

/* ------------------------------------------------- two-phase form of mul_mat
 * ggml's CPU mul_mat first converts all of src1 to Q8_0 into its work buffer
 * (from_float into params->wdata), then runs the dots.  The same two phases
 * as separate calls: one prepared activation can feed several mul_mats that
 * share an input (the q / k / v row views of one fused qkv weight,
 * cpp_ggml/src/ss_flow_graph.cpp:241-245), and each kernel can be timed alone.
 * The prepared buffer holds int8 codes [m][k] and fp32 scales [k/32][ldm]. */
B2Q_API size_t b2q_act_prepared_size(int64_t m, int64_t k);
B2Q_API int b2q_act_prepare(const float* x, int64_t m, int64_t k, int64_t x_row_stride_bytes,
                            int variant, void* act, size_t act_bytes, void* stream);
B2Q_API int b2q_mul_mat_prepared(const void* packed, int64_t n, int64_t k, const void* act,
                                 int64_t m, const float* bias, float* y,
                                 int64_t y_row_stride_bytes, void* stream);

/* ------------------------------------------------- compact Q4_0 weights
 * Q4_0 kept at its GGUF footprint (0.5625 bytes per value, against 1.125 for
 * the int8 layout b2q_weight_pack builds): b2q_weight_pack_q4_0 moves each
 * block's 16 nibble bytes to 16-byte-aligned rows and its fp16 scale to a
 * block-major table (b2q_weight_packed_q4_0_bytes(n, k) bytes, 256-byte
 * aligned; from GGUF Q4_0 rows as cpp_ggml/src/gguf_loader.cpp:113-133 loads
 * them, w_row_stride_bytes apart, 2-byte aligned).  The GEMM widens the nibbles
 * to int8 (value - 8) in shared memory before the MMA, so the result is the
 * same, bit for bit, as b2q_mul_mat_prepared on the b2q_weight_pack layout of
 * the same weight (ggml's CPU mul_mat semantics, Q8_0 activations from
 * b2q_act_prepare):
 *   b2q_mul_mat_prepared_q4_0: y = w.act + bias, or with resid != NULL
 *     y = resid + gate * (w.act + bias) (gate may be NULL; resid and y the same
 *     buffer with the same stride, or disjoint);
 *   b2q_mul_mat_prepared_q4_0_gelu_q8: the fused GELU + Q8_0 tile end of
 *     b2q_mul_mat_prepared_gelu_q8 (n % 32 == 0). */
B2Q_API size_t b2q_weight_packed_q4_0_bytes(int64_t n, int64_t k);
B2Q_API int b2q_weight_pack_q4_0(const void* w, int64_t n, int64_t k, int64_t w_row_stride_bytes, void* packed,
                                 size_t packed_bytes, void* stream);
B2Q_API int b2q_mul_mat_prepared_q4_0(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                      const float* bias, const float* gate, const float* resid,
                                      int64_t resid_row_stride_bytes, float* y, int64_t y_row_stride_bytes,
                                      void* stream);
B2Q_API int b2q_mul_mat_prepared_q4_0_gelu_q8(const void* packed, int64_t n, int64_t k, const void* act,
                                              int64_t m, const float* bias, void* act_out, size_t act_out_bytes,
                                              int variant, void* stream);

/* Q4_K on prepared operands: the packed Q4_K weight (b2q_weight_pack /
 * b2q_weight_upload with B2Q_TYPE_Q4_K) against Q8_K activations
 * (b2q_act_prepare with B2Q_ACT_Q8_K):
 *   y = mul_mat(w, act) + bias,  or, with resid != NULL,
 *   y = resid + gate * (mul_mat(w, act) + bias)   (gate may be NULL)
 * in ggml's roundings for the add / mul steps.  The tensor cores accumulate
 * each 256-value super-block exactly in int32 (three int8 weight planes), and
 * the fp32 fold runs once per super-block.  resid and y: the same buffer with
 * the same row stride, or disjoint. */
B2Q_API int b2q_mul_mat_prepared_q4_k(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                      const float* bias, const float* gate, const float* resid,
                                      int64_t resid_row_stride_bytes, float* y, int64_t y_row_stride_bytes,
                                      void* stream);

/* ------------------------------------- fused MLP hidden layer (fc1 -> fc2)
 * The DiT feed-forward block computes fc2(gelu(fc1(x) + b1)) + b2
 * (cpp_ggml/src/ss_flow_graph.cpp:380-384; graph_builder.cpp:191-197): two
 * mul_mats with ggml_gelu between them, and fc2's mul_mat quantizes the GELU
 * output to Q8_0 before its dot products.  This entry runs fc1 with the bias,
 * the GELU and that Q8_0 quantize fused into the GEMM's epilogue, writing
 * fc2's prepared activations (the b2q_act_prepare layout for m rows and
 * k_next = n) instead of the fp32 hidden state.  act_out then equals, byte for
 * byte on the written regions, b2q_act_prepare(gelu(b2q_mul_mat_prepared(...)))
 * with the same variant: no fp32 [m][n] tensor is written or read back.
 * GELU is ggml_gelu as the ggml CPU backend computes it (its fp16-table form:
 * 0 for x <= -10, x for x >= 10, else the tanh form at fp16(x), rounded to
 * fp16).  Requires n % 32 == 0; act_out_bytes >= b2q_act_prepared_size(m, n).
 * No single reference counterpart: it replaces the op sequence
 * ggml_mul_mat -> ggml_add -> ggml_gelu -> (next ggml_mul_mat's from_float). */
B2Q_API int b2q_mul_mat_prepared_gelu_q8(const void* packed, int64_t n, int64_t k, const void* act,
                                         int64_t m, const float* bias, void* act_out,
                                         size_t act_out_bytes, int variant, void* stream);
/* The end of a DiT branch: the output projection (attention to_out, or fc2),
 * its bias, the adaLN gate and the residual add in one GEMM:
 *   y[i][j] = resid[i][j] + gate[j] * (mul_mat(w, act)[i][j] + bias[j])
 * with ggml's roundings (ggml_add of the bias, ggml_mul by the gate, ggml_add
 * of the residual; cpp_ggml/src/ss_flow_graph.cpp:383-387 for the MLP branch).
 * gate and bias may be NULL.  resid and y are either the same buffer with the
 * same row stride (in-place update of the residual stream) or disjoint. */
B2Q_API int b2q_mul_mat_prepared_gate_residual(const void* packed, int64_t n, int64_t k, const void* act,
                                               int64_t m, const float* bias, const float* gate,
                                               const float* resid, int64_t resid_row_stride_bytes, float* y,
                                               int64_t y_row_stride_bytes, void* stream);
/* ggml_gelu (GGML_OP_UNARY, GGML_UNARY_OP_GELU) on an fp32 [rows][cols]
 * matrix, the same arithmetic as the fused epilogue above; x == y allowed. */
B2Q_API int b2q_gelu(const float* x, int64_t rows, int64_t cols, int64_t x_row_stride_bytes,
                     float* y, int64_t y_row_stride_bytes, void* stream);

/* ----------------------------------------- DiT pre-norm (LayerNorm + modulate)
 * h = ggml_norm(x, eps) (LayerNorm over each row of c values, no affine), then
 * the adaLN modulate h = (h * mod_scale + h) + mod_shift with mod_scale and
 * mod_shift per column (cpp_ggml/src/ss_flow_graph.cpp:45-53; used before
 * every self-attention and MLP branch, :200-204, :378-379; gb_layer_norm at
 * graph_builder.cpp:62-68).  Either modulation vector may be NULL (that term is
 * skipped; both NULL is plain ggml_norm).  mean and variance are accumulated in
 * double as ggml's CPU norm does.  Requires c % 32 == 0, c <= 4096, x, y and
 * the modulation vectors 16-byte aligned, row strides multiples of 16 bytes.
 * b2q_norm_modulate writes fp32 y; b2q_norm_modulate_q8 writes the next
 * mul_mat's prepared Q8_0 activations (b2q_act_prepare layout for m rows and
 * k = c), equal byte for byte to b2q_act_prepare(b2q_norm_modulate(...)). */
B2Q_API int b2q_norm_modulate(const float* x, int64_t m, int64_t c, int64_t x_row_stride_bytes, float eps,
                              const float* mod_scale, const float* mod_shift, float* y,
                              int64_t y_row_stride_bytes, void* stream);
/* gb_layer_norm with an affine weight and bias (the cross-attention's norm2,
 * cpp_ggml/src/ss_flow_graph.cpp:310-312): ggml_norm, then h * weight
 * (ggml_mul), then + bias (ggml_add), into Q8_0 prepared activations; same
 * requirements as b2q_norm_modulate_q8. */
B2Q_API int b2q_layer_norm_q8(const float* x, int64_t m, int64_t c, int64_t x_row_stride_bytes, float eps,
                              const float* weight, const float* bias, int variant, void* act, size_t act_bytes,
                              void* stream);
B2Q_API int b2q_norm_modulate_q8(const float* x, int64_t m, int64_t c, int64_t x_row_stride_bytes, float eps,
                                 const float* mod_scale, const float* mod_shift, int variant, void* act,
                                 size_t act_bytes, void* stream);

/* ------------------------------------------ DiT self-attention in and out
 * The tensors on either side of the attention core of an SS-flow block
 * (cpp_ggml/src/ss_flow_graph.cpp:206-290; graph_builder.cpp:70-175).
 *
 * b2q_qkv_heads: the fused qkv projection output, fp32 rows [B*T][3C] (C =
 * H*D, row stride qkv_row_stride_bytes) -> q, k, v as fp16 [B][H][T][D]
 * (IEEE half, round to nearest even).  q and k go through the per-head RMS
 * norm of gb_rms_norm_head (ggml_rms_norm with eps, then times gamma[h][d];
 * gamma may be NULL); v is only converted.  fp16 is the K/V form of the
 * reference's flash-attention path.  D in {32, 64, 128}.
 *
 * b2q_heads_act_prepare: an attention output o[b][h][t][d] (fp16, element
 * strides stride_b / stride_h / stride_t, d contiguous) -> the Q8_0 prepared
 * activations (b2q_act_prepare layout) of the output projection for rows
 * b*T + t and K = H*D.  D % 32 == 0. */
B2Q_API int b2q_qkv_heads(const float* qkv, int64_t B, int64_t T, int64_t H, int64_t D,
                          int64_t qkv_row_stride_bytes, const float* gamma_q, const float* gamma_k, float eps,
                          void* q16, void* k16, void* v16, void* stream);
/* The same conversion for projections without the RMS norm (the
 * cross-attention's q, and its k | v computed from the condition tokens as
 * one 2C-wide projection): `parts` (1 or 2) C-wide fp32 tensors per row ->
 * fp16 [B][H][T][D] each (out1 used when parts == 2). */
B2Q_API int b2q_rows_to_heads(const float* src, int64_t B, int64_t T, int64_t H, int64_t D, int parts,
                              int64_t src_row_stride_bytes, void* out0, void* out1, void* stream);
/* b2q_mul_mat_prepared (+ bias) with the head layout as its tile end: the
 * cross-attention's q projection (parts = 1) or its fused k | v projection of
 * the condition tokens (parts = 2) straight into fp16 [B][H][T][64] heads
 * (cpp_ggml/src/ss_flow_graph.cpp:297-345: ggml_mul_mat + ggml_add, then the
 * reshape / permute / cast to F16 that gb_attention's flash path reads,
 * graph_builder.cpp:151-171).  n = parts*H*64, m = B*T; each output is the fp32
 * value b2q_mul_mat_prepared writes, rounded once to fp16, so the bytes equal
 * b2q_mul_mat_prepared followed by b2q_rows_to_heads.  D other than 64 and
 * m <= 8 (the few-token path; use the two calls) return B2Q_ERR_UNSUPPORTED;
 * packed and act 256-byte aligned, out0 / out1 2-byte aligned. */
B2Q_API int b2q_mul_mat_prepared_heads_f16(const void* packed, int64_t n, int64_t k, const void* act, int64_t m,
                                           const float* bias, int64_t B, int64_t T, int64_t H, int64_t D,
                                           int parts, void* out0, void* out1, void* stream);
B2Q_API int b2q_heads_act_prepare(const void* o16, int64_t B, int64_t T, int64_t H, int64_t D, int64_t stride_b,
                                  int64_t stride_h, int64_t stride_t, int variant, void* act, size_t act_bytes,
                                  void* stream);

/* ------------------------------------------------ attention, F32 contract
 * The numeric-gate form of gb_attention (cpp_ggml/src/graph_builder.cpp:
 * 139-175 with AttentionOptions.strict_kv: ggml_flash_attn_ext on F32 Q, K and
 * V with GGML_PREC_F32), the form the reference keeps for parity diagnosis:
 *   o[b*Tq + t][h*D + d] = sum_j p_j v[b][h][j][d] / sum_j p_j,
 *   p_j = exp(s_j - max_j s_j),  s_j = scale * (q[b][h][t] . key_j)
 * as a per-query online softmax with every product, sum and exp in IEEE fp32.
 * q fp32 [B][H][Tq][D]; k, v fp32 [B][H][Tk][D]; an optional second key source
 * k2, v2 fp32 [B][H][Tk2][D] supplies keys Tk .. Tk + Tk2 - 1 (the pose group
 * attends its own keys followed by the shape group's,
 * cpp_ggml/src/ss_flow_graph.cpp:262-275); both NULL for none.  o is written as
 * fp32 rows [B*Tq] of o_row_stride_bytes, head h at columns h*D .. h*D+D-1: the
 * [D, H, Tq, B] tensor the output projection reads (graph_builder.cpp:
 * 146-149).  D in {32, 64, 128}; q, k, v, k2, v2 16-byte aligned.
 * b2q_qkv_heads_f32 / b2q_rows_to_heads_f32 are b2q_qkv_heads /
 * b2q_rows_to_heads with fp32 outputs (no fp16 rounding), the inputs of this
 * form; outputs 16-byte aligned. */
/* ------------------------------------------------- attention, F16 (production)
 * gb_attention's production path (cpp_ggml/src/graph_builder.cpp:151-171:
 * ggml_flash_attn_ext with K and V cast to F16) for D = 64, on the tensor cores:
 * S = q k^T (fp16 x fp16, fp32 accumulation), softmax in fp32 (exp2 of the
 * scores times scale * log2 e), P rounded to fp16, o = P v / sum P in fp32,
 * o rounded to fp16.  q fp16 [B][H][Tq][64]; k, v fp16 [B][H][Tk][64]; optional
 * k2, v2 [B][H][Tk2][64] append keys Tk .. Tk + Tk2 - 1 (both NULL for none).
 * o is written as fp16 rows [B*Tq] of o_row_stride_bytes (a multiple of 16),
 * head h at columns h*64 .. h*64+63 -- b2q_heads_act_prepare reads it with
 * strides (Tq*row, 64, row).  All pointers 16-byte aligned.  D other than 64
 * returns B2Q_ERR_UNSUPPORTED. */
B2Q_API int b2q_attention_f16(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t Tq,
                              int64_t Tk, int64_t D, const void* k2, const void* v2, int64_t Tk2, float scale,
                              void* o, int64_t o_row_stride_bytes, void* stream);
/* b2q_attention_f16 with the output going straight into the output projection's
 * Q8_0 prepared activations (b2q_act_prepare layout, rows b*Tq + t, K = H*64,
 * act 256-byte aligned, act_bytes >= b2q_act_prepared_size(B*Tq, H*64)): each
 * output is rounded to fp16 as b2q_attention_f16 stores it and quantized with
 * `variant`'s arithmetic, so the bytes equal b2q_attention_f16 followed by
 * b2q_heads_act_prepare (the self- and cross-attention outputs of
 * cpp_ggml/src/ss_flow_graph.cpp:277-289 and 346-349 feeding their to_out linears). */
B2Q_API int b2q_attention_f16_q8(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t Tq,
                                 int64_t Tk, int64_t D, const void* k2, const void* v2, int64_t Tk2, float scale,
                                 int variant, void* act, size_t act_bytes, void* stream);
B2Q_API int b2q_qkv_heads_f32(const float* qkv, int64_t B, int64_t T, int64_t H, int64_t D,
                              int64_t qkv_row_stride_bytes, const float* gamma_q, const float* gamma_k, float eps,
                              float* q, float* k, float* v, void* stream);
B2Q_API int b2q_rows_to_heads_f32(const float* src, int64_t B, int64_t T, int64_t H, int64_t D, int parts,
                                  int64_t src_row_stride_bytes, float* out0, float* out1, void* stream);
B2Q_API int b2q_attention_f32(const float* q, const float* k, const float* v, int64_t B, int64_t H, int64_t Tq,
                              int64_t Tk, int64_t D, const float* k2, const float* v2, int64_t Tk2, float scale,
                              float* o, int64_t o_row_stride_bytes, void* stream);

/* ----------------------------------------- dequantize-to-float form (strict)
 * matmul_weight with keep_quant_gemm false (cpp_ggml/src/ss_flow_graph.cpp:
 * 13-34, slat_flow_graph.cpp:89-94): the quantized weight is cast to F32
 * (as_f32) or to F32 then F16 (as_f16) with ggml_cast, and gb_linear
 * (graph_builder.cpp:44-60) multiplies with GGML_PREC_F32.
 *
 * b2q_dequantize: n GGUF rows of wtype (Q8_0, Q4_0, Q4_K; w_row_stride_bytes
 * apart, 2-byte aligned) -> [n][k] out_type (B2Q_TYPE_F32 or B2Q_TYPE_F16) rows
 * out_row_stride_bytes apart (16-byte aligned).  Values as ggml's
 * dequantize_row_*: Q8_0 / Q4_0 fp32(d) * code (Q4_0 code - 8); Q4_K
 * (d * sc) * q - (dmin * m), each product and the difference rounded once;
 * F16 by one round-to-nearest-even of that fp32 value.  k % 32 == 0 (Q4_K:
 * k % 256 == 0).
 *
 * b2q_mul_mat_f32: the strict F32 mul_mat, y[m][n] = sum_k x[m][k] * w[n][k]
 * (+ bias[n], one more rounding: ggml's separate ADD) -- F32 weights (the
 * as_f32 result) times F32 activations with every product and sum in fp32
 * (one FMA chain per output, in k order; the CUDA cores, no tensor-core
 * rounding).  w, x 16-byte aligned with row strides multiples of 16 bytes,
 * k % 4 == 0; y 4-byte aligned.  The as_f16 form is b2q_dequantize(...,
 * B2Q_TYPE_F16, ...) followed by b2q_mul_mat with wtype B2Q_TYPE_F16. */
B2Q_API int b2q_dequantize(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n, int64_t k,
                           int out_type, void* out, int64_t out_row_stride_bytes, void* stream);
B2Q_API int b2q_mul_mat_f32(const float* w, int64_t w_row_stride_bytes, int64_t n, int64_t k, const float* x,
                            int64_t x_row_stride_bytes, int64_t m, const float* bias, float* y,
                            int64_t y_row_stride_bytes, void* stream);

/* ------------------------------------------- column-parallel form (multi-GPU)
 * One rank of a tensor-parallel group for a single large mul_mat (the SLat
 * flow transformer's linears at 8k-20k tokens): the weight is split by output
 * rows across the ranks and every rank needs the full [M][N_total] output.
 * This rank holds the packed rows [y_col0, y_col0 + n) of the weight and writes
 * its output columns straight into the full-width y buffer of EVERY rank:
 * y_peers[q] (host array of n_peers <= 8 device pointers this GPU can store to:
 * its own buffer and its peers' through CUDA IPC / peer access over NVLink),
 * element (m, j) to y_peers[q][m * y_row_stride_bytes/4 + y_col0 + j].  That is
 * the GEMM and the all-gather of its outputs in one kernel, each tile leaving
 * over NVLink while the next tiles compute.  No counterpart in the reference
 * (it runs one process per GPU with no tensor parallelism); it replaces the
 * column-parallel plan "ggml_mul_mat on a weight row slice, then ncclAllGather
 * and a [P][M][N/P] -> [M][N] transpose".  The call only launches: the ranks
 * must synchronise (every rank's kernel complete) before any rank reads y. */
B2Q_API int b2q_mul_mat_prepared_peers(const void* packed, int64_t n, int64_t k, const void* act,
                                       int64_t m, const float* bias, float* const* y_peers,
                                       int n_peers, int64_t y_col0, int64_t y_row_stride_bytes,
                                       void* stream);

/* Column-parallel form of b2q_mul_mat_prepared_gelu_q8: the exchange is the
 * next layer's Q8_0 input (1.125 bytes per value over NVLink instead of 4).
 * This rank holds the packed rows [col0, col0 + n) of the weight (n and col0
 * multiples of 32, col0 + n <= n_total); it writes quantize_q8_0(gelu(w.x +
 * bias)) of those output columns, which are the next layer's activation
 * columns [col0, col0 + n), into EVERY rank's prepared-activation buffer:
 * act_peers[q] (n_peers <= 8 device pointers, 256-byte aligned, each
 * act_bytes >= b2q_act_prepared_size(m, n_total) long, this rank's own and
 * its peers' CUDA-IPC mappings).  Once every rank's kernel is complete each
 * buffer holds b2q_act_prepare(gelu(x . W^T + b)) of the whole weight,
 * bit-identical to the single-GPU b2q_mul_mat_prepared_gelu_q8; the next
 * mul_mat reads it directly.  Launch only: the ranks synchronise before any
 * rank reads the buffers.  No counterpart in the reference (one process per
 * GPU, no tensor parallelism). */
B2Q_API int b2q_mul_mat_prepared_gelu_q8_peers(const void* packed, int64_t n, int64_t k, const void* act,
                                               int64_t m, const float* bias, void* const* act_peers,
                                               int n_peers, int64_t n_total, int64_t col0, size_t act_bytes,
                                               int variant, void* stream);

/* ------------------------------------------------------------ debug / check
 * int32 per-block dot products S_b computed by the tensor-core GEMM itself
 * (the value its epilogue reads from tensor memory), for parity checks:
 *   dots[(m*n_rows + n)*(k/32) + b] = S_b(weight row n, activation row m).
 * a: Q8_0 activation blocks (ggml layout, a_row_stride_bytes apart).
 * Requires m*n*(k/32) <= 2^28.  No counterpart exists in ggml (its vec_dot
 * keeps S_b in registers); this exposes the int8 MMA's exact results. */
B2Q_API int b2q_block_dots(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n, int64_t k,
                   const void* a, int64_t m, int64_t a_row_stride_bytes, int32_t* dots,
                   void* workspace, size_t workspace_bytes, void* stream);
B2Q_API size_t b2q_block_dots_workspace_size(int64_t m, int64_t n, int64_t k);

/* Plain CUDA-core kernel with ggml's x86 accumulation order (8 fp32 lanes of
 * 4-product int32 partials, pairwise lane reduction): bit-exact fp32 output
 * for the CPU backend's mul_mat on pre-quantized activations.  A reference
 * path for checks, not a fast path.  a: Q8_0 activation blocks. */
B2Q_API int b2q_mul_mat_q_simt(int wtype, const void* w, int64_t w_row_stride_bytes, int64_t n,
                       int64_t k, const void* a, int64_t m, int64_t a_row_stride_bytes,
                       float* y, int64_t y_row_stride_bytes, void* stream);

/* ------------------------------------------------------ SLat sparse stages
 * b2q_sparse_conv_f16: the F16 submanifold convolution of the SLat flow
 * transformer, ggml_sam3d_sparse_conv_f16 (ggml patch
 * 0001-sam3d-ggml-combined.patch:65-76 declaration, :217-272 CPU semantics;
 * called at cpp_ggml/src/slat_flow_graph.cpp:168-221):
 *   y16[t][n] = fp16(bias[n] + sum_{o<27} sum_{c<C} w16[n][o*C + c] * x16[idx[o*tokens + t]][c])
 * with fp32 accumulation; a neighbour index < 0 or >= tokens contributes
 * nothing (the reference's -1 / sentinel row).  x16 fp16 [tokens][C]; w16 fp16
 * [Cout][27*C] (the converter's row format); bias16 fp16 [Cout] or NULL; idx
 * int32 [27][tokens], offset-major; y16 fp16 [tokens][Cout].  Runs a gather of
 * the 27 neighbour rows into the workspace, then the kind::f16 tensor-core
 * GEMM with K = 27*C and an fp16 epilogue.  C % 8 == 0; x16 and w16 16-byte
 * aligned; workspace 256-byte aligned, b2q_sparse_conv_f16_workspace_bytes.
 *
 * b2q_sparse_scatter_mean_f16: the SLat 2x downsample,
 * ggml_sam3d_sparse_scatter_mean (patch :55-63 declaration, :151-215 CPU
 * semantics; slat_flow_graph.cpp:223-236): out16 [coarse][C] = every fine row i
 * with 0 <= rows[i] < coarse added into out16[rows[i]] in ascending i, each
 * partial sum rounded to fp16, starting from zero; then each value divided in
 * fp32 by counts[c] (|children| + 1 in the reference) and rounded to fp16.
 * Bit-exact with that CPU path.  C % 8 == 0; features16 and out16 16-byte
 * aligned; workspace b2q_sparse_scatter_mean_workspace_bytes. */
B2Q_API size_t b2q_sparse_conv_f16_workspace_bytes(int64_t tokens, int64_t channels, int64_t out_channels);
B2Q_API int b2q_sparse_conv_f16(const void* x16, int64_t tokens, int64_t channels, const void* w16,
                                int64_t out_channels, const void* bias16, const int32_t* indices, void* y16,
                                void* workspace, size_t workspace_bytes, void* stream);
/* Planned form of b2q_sparse_conv_f16 for a neighbour table that serves many
 * calls (the SLat tables are built once per object and reused by every
 * sampling step).  The dense form multiplies all 27 neighbour slots, empty
 * ones included, as the reference's get_rows + GEMM does; at the sparse
 * occupancies of SLat most slots are empty.  b2q_sparse_conv_plan lists the
 * occupied (output token, input token) pairs of every offset, in token order,
 * padded per offset to 256-row tiles (plan of b2q_sparse_conv_plan_bytes(tokens)
 * bytes, 16-byte aligned).  b2q_sparse_conv_f16_planned then gathers only those
 * rows, runs one grouped kind::f16 GEMM in which every tile multiplies its
 * offset's weight slice W_o, and sums each token's partials in fp32 in offset
 * order onto the bias before the fp16 rounding: the same result as
 * b2q_sparse_conv_f16 within fp32 summation order.  channels % 64 == 0,
 * out_channels % 8 == 0; x16, w16, y16 16-byte aligned; workspace
 * b2q_sparse_conv_f16_planned_workspace_bytes (sized for any table of that
 * many tokens).  The plan stays valid while the table does not change. */
B2Q_API size_t b2q_sparse_conv_plan_bytes(int64_t tokens);
B2Q_API int b2q_sparse_conv_plan(const int32_t* indices, int64_t tokens, void* plan, size_t plan_bytes, void* stream);
B2Q_API size_t b2q_sparse_conv_f16_planned_workspace_bytes(int64_t tokens, int64_t channels, int64_t out_channels);
B2Q_API int b2q_sparse_conv_f16_planned(const void* x16, int64_t tokens, int64_t channels, const void* w16,
                                        int64_t out_channels, const void* bias16, const void* plan, void* y16,
                                        void* workspace, size_t workspace_bytes, void* stream);
B2Q_API size_t b2q_sparse_scatter_mean_workspace_bytes(int64_t fine_rows, int64_t coarse_rows);
B2Q_API int b2q_sparse_scatter_mean_f16(const void* features16, int64_t fine_rows, int64_t channels,
                                        const int32_t* row_indices, const float* counts, int64_t coarse_rows,
                                        void* out16, void* workspace, size_t workspace_bytes, void* stream);
/* The same in two parts, for a mapping that serves many calls (the SLat
 * downsample table is fixed per object, cpp_ggml/src/slat_flow_graph.cpp:
 * 223-236, and reused by every sampling step): b2q_sparse_scatter_plan lists the
 * fine rows of every coarse row in ascending order into `plan`
 * (b2q_sparse_scatter_mean_workspace_bytes(fine, coarse) bytes, 4-byte
 * aligned); b2q_sparse_scatter_mean_f16_planned then runs the accumulation
 * alone, one launch, bit-identical to b2q_sparse_scatter_mean_f16.  The plan
 * stays valid while row_indices, fine_rows and coarse_rows do not change. */
B2Q_API int b2q_sparse_scatter_plan(const int32_t* row_indices, int64_t fine_rows, int64_t coarse_rows, void* plan,
                                    size_t plan_bytes, void* stream);
B2Q_API int b2q_sparse_scatter_mean_f16_planned(const void* features16, int64_t fine_rows, int64_t channels,
                                                const void* plan, const float* counts, int64_t coarse_rows,
                                                void* out16, void* stream);

/* Fault-free test of the failure path: launches the GEMM of
 * b2q_mul_mat_prepared with its TMA producer withholding every stage, so the
 * MMA and epilogue waits run out (after ~2 s), the kernel drains, frees its
 * tensor memory and ends, and b2q_device_status then returns B2Q_ERR_DEVICE
 * with the code of the wait that gave up.  y is not written.  Nothing faults,
 * traps or hangs; the context stays usable.  No counterpart in the reference
 * (its failures are bool returns and aborting asserts). */
B2Q_API int b2q_selftest_stalled_mul_mat(const void* packed, int64_t n, int64_t k, const void* act,
                                         int64_t m, float* y, int64_t y_row_stride_bytes, void* stream);

/* Device status word written by kernels whose bounded waits gave up:
 * *code = 0 when none; clear != 0 resets it.  Synchronises the device. */
B2Q_API int b2q_device_status(unsigned int* code, int clear);

#ifdef __cplusplus
}
#endif

#endif /* B2Q_H */
