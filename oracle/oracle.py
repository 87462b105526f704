"""ctypes view of the CPU oracle (``oracle/_build/libb2q_oracle.so``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` as the
checker.  The product library never loads it.

The oracle restates ggml's Q8_0 / Q4_0 ``GGML_OP_MUL_MAT`` on the CPU backend
(ggml v0.21.0, pinned by the reference at cpp_ggml/CMakeLists.txt:126; the
submodule is empty in the reference checkout).  Weight quantizers and the
scalar Q8_0 quantizer are pinned byte-for-byte against gguf-py 0.19.0
(``gguf.quants``), the reference converter's dependency
(cpp_ggml/scripts/gguf_schema.py:11, cpp_ggml/scripts/gguf_torch_loader.py:26).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libb2q_oracle.so")

QK = 32
TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0, TYPE_Q4_K = 0, 1, 2, 8, 12
QK_K, Q4_K_BYTES, Q8_K_BYTES = 256, 144, 292
ACT_X86, ACT_REF = 0, 1
BLOCK_BYTES = {TYPE_Q8_0: 34, TYPE_Q4_0: 18}

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.b2q_orc_fp32_to_fp16.restype = ctypes.c_uint16
        L.b2q_orc_fp32_to_fp16.argtypes = [ctypes.c_float]
        L.b2q_orc_fp16_to_fp32.restype = ctypes.c_float
        L.b2q_orc_fp16_to_fp32.argtypes = [ctypes.c_uint16]
        L.b2q_orc_fp32_to_fp16_n.argtypes = [P, P, I64]
        L.b2q_orc_quantize_rows.argtypes = [I, P, P, I64, I64, I]
        L.b2q_orc_dequantize_row.argtypes = [I, P, P, I64]
        L.b2q_orc_vec_dot.restype = ctypes.c_float
        L.b2q_orc_vec_dot.argtypes = [I, P, P, I64]
        L.b2q_orc_block_dots.argtypes = [I, P, I64, I64, P, I64, I64, I64, P]
        L.b2q_orc_mul_mat_q.argtypes = [I, P, I64, I64, P, I64, I64, I64, P, I64, I]
        L.b2q_orc_mul_mat.argtypes = [I, P, I64, I64, P, I64, I64, I64, I, P, I64, I]
        L.b2q_orc_mul_mat.restype = I
        L.b2q_orc_mul_mat_q_fast.argtypes = [I, P, I64, I64, P, I64, I64, I64, P, I64, I]
        L.b2q_orc_mul_mat_q_fast.restype = I
        L.b2q_orc_mul_mat_fast.argtypes = [I, P, I64, I64, P, I64, I64, I64, I, P, I64, I]
        L.b2q_orc_mul_mat_fast.restype = I
        L.b2q_orc_mul_mat_f64.argtypes = [I, P, I64, I64, P, I64, I64, I64, P]
        L.b2q_orc_philox4x32_10.argtypes = [ctypes.c_uint64, ctypes.c_uint64, P]
        L.b2q_orc_fill_normal.argtypes = [P, I64, ctypes.c_uint64, ctypes.c_float, ctypes.c_float]
        L.b2q_orc_gelu.restype = ctypes.c_float
        L.b2q_orc_gelu.argtypes = [ctypes.c_float, I]
        L.b2q_orc_gelu_n.argtypes = [P, P, I64, I]
        L.b2q_orc_gelu_table.argtypes = [P, I]
        L.b2q_orc_norm_modulate.argtypes = [P, I64, I64, I64, ctypes.c_float, P, P, P, I64]
        L.b2q_orc_dequantize_row_q4_K.argtypes = [P, P, I64]
        L.b2q_orc_quantize_row_q8_K.argtypes = [P, P, I64]
        L.b2q_orc_vec_dot_q4_K_q8_K.restype = ctypes.c_float
        L.b2q_orc_vec_dot_q4_K_q8_K.argtypes = [P, P, I64]
        L.b2q_orc_mul_mat_q4_K.argtypes = [P, I64, I64, P, I64, I64, I64, P, I64, I]
        L.b2q_orc_mul_mat_q4_K.restype = I
        L.b2q_orc_num_threads.restype = I
        L.b2q_orc_isa.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def fp32_to_fp16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().b2q_orc_fp32_to_fp16_n(_p(x), _p(out), x.size)
    return out


def quantize(x: np.ndarray, wtype: int, act_variant: int | None = None) -> np.ndarray:
    """Quantize rows of ``x`` [rows, K] into ggml blocks [rows, K/32*bytes] (uint8).

    ``act_variant`` None -> the ggml reference quantizer (weights);
    ACT_X86 / ACT_REF -> the activation quantizer variant (Q8_0 only).
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, k = x.shape
    assert k % QK == 0
    out = np.empty((rows, k // QK * BLOCK_BYTES[wtype]), dtype=np.uint8)
    v = -1 if act_variant is None else int(act_variant)
    lib().b2q_orc_quantize_rows(wtype, _p(x), _p(out), rows, k, v)
    return out


def dequantize(q: np.ndarray, wtype: int, k: int) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    rows = q.shape[0]
    out = np.empty((rows, k), dtype=np.float32)
    for r in range(rows):
        lib().b2q_orc_dequantize_row(wtype, _p(q[r]), _p(out[r]), k)
    return out


def block_dots(wtype: int, w: np.ndarray, a: np.ndarray, K: int) -> np.ndarray:
    """int32 [M, N, K/32]: per-block dot products of weight rows and Q8_0 activation rows."""
    w = np.ascontiguousarray(w)
    a = np.ascontiguousarray(a)
    N, M = w.shape[0], a.shape[0]
    out = np.empty((M, N, K // QK), dtype=np.int32)
    lib().b2q_orc_block_dots(wtype, _p(w), w.shape[1], N, _p(a), a.shape[1], M, K, _p(out))
    return out


def mul_mat_q(wtype: int, w: np.ndarray, a: np.ndarray, K: int, nthreads: int = 0,
              fast: bool = False) -> np.ndarray:
    """Y [M, N] fp32 from weight blocks [N, .] and Q8_0 activation blocks [M, .]."""
    w = np.ascontiguousarray(w)
    a = np.ascontiguousarray(a)
    N, M = w.shape[0], a.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    fn = lib().b2q_orc_mul_mat_q_fast if fast else lib().b2q_orc_mul_mat_q
    fn(wtype, _p(w), w.shape[1], N, _p(a), a.shape[1], M, K, _p(y), N, nthreads)
    return y


def mul_mat(wtype: int, w: np.ndarray, x: np.ndarray, act_variant: int = ACT_X86,
            nthreads: int = 0, fast: bool = True) -> np.ndarray:
    """GGML_OP_MUL_MAT(src0 = w blocks [N, .], src1 = x fp32 [M, K]) -> [M, N] fp32."""
    w = np.ascontiguousarray(w)
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    fn = lib().b2q_orc_mul_mat_fast if fast else lib().b2q_orc_mul_mat
    rc = fn(wtype, _p(w), w.shape[1], N, _p(x), K, M, K, act_variant, _p(y), N, nthreads)
    if rc < 0:
        raise MemoryError("oracle mul_mat failed to allocate")
    return y


def mul_mat_f16(w16: np.ndarray, x: np.ndarray) -> np.ndarray:
    """GGML_OP_MUL_MAT with src0 F16 on ggml's CPU backend (the F16 GGUF
    tensors and the autocast linears, cpp_ggml/src/slat_flow_graph.cpp:29-40;
    exercised by cpp_ggml/src/matmul_backend_test.cpp:177-183): src1 is rounded
    to fp16 (vec_dot_type F16, round to nearest even), and each output is one
    dot of fp16 x fp16 products (exact in fp32) summed in wide precision
    (ggml_vec_dot_f16 accumulates in fp32 SIMD lanes and a double; this fp64
    sum differs from it by far less than the 1e-5 parity bar) -> fp32."""
    x16 = np.asarray(x, dtype=np.float32).astype(np.float16)
    w = np.asarray(w16, dtype=np.float16)
    return (x16.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


def sparse_scatter_mean_f16(x16: np.ndarray, rows: np.ndarray, counts: np.ndarray, coarse: int) -> np.ndarray:
    """ggml_sam3d_sparse_scatter_mean on ggml's CPU backend (ggml patch
    0001-sam3d-ggml-combined.patch:151-215): out starts at fp16 zero; fine rows
    in ascending order add into their coarse row, each partial sum
    fp16(fp32(acc) + fp32(x)); rows outside [0, coarse) are skipped; finally
    fp16(fp32(acc) / counts[c])."""
    x16 = np.asarray(x16, dtype=np.float16)
    out = np.zeros((coarse, x16.shape[1]), dtype=np.float16)
    with np.errstate(over="ignore"):  # fp16 partial sums may saturate to inf, as in the reference
        for i, c in enumerate(np.asarray(rows)):
            if 0 <= c < coarse:
                out[c] = (out[c].astype(np.float32) + x16[i].astype(np.float32)).astype(np.float16)
    return (out.astype(np.float32) / np.asarray(counts, np.float32)[:, None]).astype(np.float16)


def sparse_conv_f16(x16: np.ndarray, w16: np.ndarray, b16, idx: np.ndarray) -> np.ndarray:
    """ggml_sam3d_sparse_conv_f16 on ggml's CPU backend (patch :217-272): per
    token and output channel, acc = fp32(bias), then for offset o = 0..26 and
    channel c in order acc += fp32(w[n][o*C + c]) * fp32(x[idx[o][t]][c]) in
    fp32 (the product of two fp16 values is exact in fp32, so a fused or
    separate multiply-add gives the same sum), skipping indices outside
    [0, tokens); result fp16(acc).  Vectorised over tokens and outputs, in the
    reference's summation order."""
    x16 = np.asarray(x16, dtype=np.float16)
    w16 = np.asarray(w16, dtype=np.float16)
    tokens, C = x16.shape
    cout = w16.shape[0]
    w = w16.astype(np.float32).reshape(cout, 27, C)
    x = x16.astype(np.float32)
    acc = np.zeros((tokens, cout), np.float32) if b16 is None else np.tile(
        np.asarray(b16, np.float16).astype(np.float32), (tokens, 1))
    for o in range(27):
        src = np.asarray(idx)[o]
        ok = (src >= 0) & (src < tokens)
        xs = np.zeros((tokens, C), np.float32)
        xs[ok] = x[src[ok]]
        for c in range(C):
            acc += (xs[:, c][:, None] * w[:, o, c][None, :]).astype(np.float32)
    return acc.astype(np.float16)


def mul_mat_f64(wtype: int, w: np.ndarray, a: np.ndarray, K: int) -> np.ndarray:
    w = np.ascontiguousarray(w)
    a = np.ascontiguousarray(a)
    N, M = w.shape[0], a.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    lib().b2q_orc_mul_mat_f64(wtype, _p(w), w.shape[1], N, _p(a), a.shape[1], M, K, _p(y))
    return y


def philox(seed: int, counter: int) -> np.ndarray:
    out = np.empty(4, dtype=np.uint32)
    lib().b2q_orc_philox4x32_10(seed, counter, _p(out))
    return out


def normal(n: int, seed: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().b2q_orc_fill_normal(_p(out), n, seed, mean, std)
    return out


def num_threads() -> int:
    return lib().b2q_orc_num_threads()


def isa() -> str:
    return lib().b2q_orc_isa().decode()


def gelu(x: np.ndarray, contract: bool = False) -> np.ndarray:
    """ggml_gelu (CPU backend, fp16-table build) elementwise; see b2q_oracle.h."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().b2q_orc_gelu_n(_p(x), _p(y), x.size, int(contract))
    return y


def gelu_table(contract: bool = False) -> np.ndarray:
    """The 65536 fp16 table entries (uint16 bits), indexed by the fp16 input bits."""
    t = np.empty(65536, dtype=np.uint16)
    lib().b2q_orc_gelu_table(_p(t), int(contract))
    return t


def norm_modulate(x: np.ndarray, eps: float = 1e-6, scale=None, shift=None) -> np.ndarray:
    """ggml_norm then h*(1+scale)+shift per column; see b2q_oracle.h."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, c = x.shape
    y = np.empty_like(x)
    sc = None if scale is None else np.ascontiguousarray(scale, dtype=np.float32)
    sh = None if shift is None else np.ascontiguousarray(shift, dtype=np.float32)
    lib().b2q_orc_norm_modulate(_p(x), m, c, c, eps, None if sc is None else _p(sc),
                                None if sh is None else _p(sh), _p(y), c)
    return y


# ------------------------------------------------------------ Q4_K / Q8_K
def random_q4_k(n: int, k: int, seed: int) -> np.ndarray:
    """Random valid Q4_K rows, uint8 [n, k/256*144]: d, dmin ~ |N(0, 0.01)| as
    fp16, random 6-bit scales and mins, random 4-bit quants (weights are
    quantized offline; any block bytes are a valid weight)."""
    rng = np.random.default_rng(seed)
    nb = k // QK_K
    b = rng.integers(0, 256, size=(n, nb, Q4_K_BYTES), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n, nb)) * 0.01).astype(np.float16)
    dm = np.abs(rng.standard_normal((n, nb)) * 0.01).astype(np.float16)
    b[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    b[:, :, 2:4] = dm.view(np.uint8).reshape(n, nb, 2)
    return b.reshape(n, nb * Q4_K_BYTES)


def dequantize_q4_k(w: np.ndarray, k: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.empty((w.shape[0], k), dtype=np.float32)
    for r in range(w.shape[0]):
        lib().b2q_orc_dequantize_row_q4_K(_p(w[r]), _p(out[r]), k)
    return out


def quantize_q8_k(x: np.ndarray) -> np.ndarray:
    """fp32 [M, K] -> Q8_K rows uint8 [M, K/256*292]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    out = np.empty((m, k // QK_K * Q8_K_BYTES), dtype=np.uint8)
    for r in range(m):
        lib().b2q_orc_quantize_row_q8_K(_p(x[r]), _p(out[r]), k)
    return out


def mul_mat_q4_k(w: np.ndarray, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, (m, k) = w.shape[0], x.shape
    y = np.empty((m, n), dtype=np.float32)
    lib().b2q_orc_mul_mat_q4_K(_p(w), w.shape[1], n, _p(x), k, m, k, _p(y), n, nthreads)
    return y
