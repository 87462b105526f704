"""Python view of libb2q's C ABI (include/b2q.h) for tests and the benchmark.

The product is the C-ABI shared library ``lib/libb2q.so``; this module binds it
with ctypes and uses torch only for device memory and streams.  Function names
and argument meaning follow the C ABI, which in turn follows ggml's
``ggml_mul_mat(ctx, w, x)`` contract (cpp_ggml/src/graph_builder.cpp:44-60):
``w`` is a [N, K] block-quantized weight (rows of ggml blocks), ``x`` a [M, K]
fp32 activation, the result ``y`` is [M, N] fp32.

There is no fallback: if the library is missing or the device is not sm_100,
every call raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libb2q.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "b2q.h")

TYPE_F32, TYPE_F16, TYPE_Q4_0, TYPE_Q8_0, TYPE_Q4_K = 0, 1, 2, 8, 12
ACT_X86, ACT_REF, ACT_Q8_K = 0, 1, 2
QK, QK_K = 32, 256
BLOCK_BYTES = {TYPE_Q8_0: 34, TYPE_Q4_0: 18}
GEMV_MAX_M = 8  # token counts up to this run on the CUDA-core few-token kernel

OK = 0
STATUS = {
    0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "MISALIGNED", 4: "WORKSPACE",
    5: "CUDA", 6: "DEVICE", 7: "TOO_LARGE",
}


class B2QError(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {STATUS.get(status, status)} ({_lib_obj().b2q_status_string(status).decode()})")


_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def _lib_obj():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is not built (run __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
        sig = {
            "b2q_status_string": (ctypes.c_char_p, [I]),
            "b2q_version": (ctypes.c_char_p, []),
            "b2q_quantize_q8_0": (I, [P, I64, I64, I64, P, I64, I, P]),
            "b2q_weight_packed_size": (SZ, [I64, I64]),
            "b2q_weight_packed_bytes": (SZ, [I, I64, I64]),
            "b2q_act_prepared_bytes": (SZ, [I, I64, I64]),
            "b2q_mul_mat_workspace_bytes": (SZ, [I, I64, I64, I64, I]),
            "b2q_mul_mat_prepared_q4_k": (I, [P, I64, I64, P, I64, P, P, P, I64, P, I64, P]),
            "b2q_weight_packed_q4_0_bytes": (SZ, [I64, I64]),
            "b2q_weight_pack_q4_0": (I, [P, I64, I64, I64, P, SZ, P]),
            "b2q_mul_mat_prepared_q4_0": (I, [P, I64, I64, P, I64, P, P, P, I64, P, I64, P]),
            "b2q_mul_mat_prepared_q4_0_gelu_q8": (I, [P, I64, I64, P, I64, P, P, SZ, I, P]),
            "b2q_weight_pack": (I, [I, P, I64, I64, I64, P, SZ, P]),
            "b2q_weight_upload": (I, [I, P, I64, I64, I64, P, SZ, P, SZ, P]),
            "b2q_mul_mat_workspace_size": (SZ, [I64, I64, I64, I]),
            "b2q_mul_mat": (I, [I, P, I64, I64, I64, P, I64, I64, P, P, I64, I, P, SZ, P]),
            "b2q_mul_mat_packed": (I, [P, I64, I64, P, I64, I64, P, P, I64, I, P, SZ, P]),
            "b2q_mul_mat_packed_noalloc": (I, [P, I64, I64, P, I64, I64, P, P, I64, I, P]),
            "b2q_act_prepared_size": (SZ, [I64, I64]),
            "b2q_act_prepare": (I, [P, I64, I64, I64, I, P, SZ, P]),
            "b2q_mul_mat_prepared": (I, [P, I64, I64, P, I64, P, P, I64, P]),
            "b2q_mul_mat_prepared_gelu_q8": (I, [P, I64, I64, P, I64, P, P, SZ, I, P]),
            "b2q_gelu": (I, [P, I64, I64, I64, P, I64, P]),
            "b2q_qkv_heads": (I, [P, I64, I64, I64, I64, I64, P, P, ctypes.c_float, P, P, P, P]),
            "b2q_heads_act_prepare": (I, [P, I64, I64, I64, I64, I64, I64, I64, I, P, SZ, P]),
            "b2q_rows_to_heads": (I, [P, I64, I64, I64, I64, I, I64, P, P, P]),
            "b2q_mul_mat_prepared_heads_f16": (I, [P, I64, I64, P, I64, P, I64, I64, I64, I64, I, P, P, P]),
            "b2q_qkv_heads_f32": (I, [P, I64, I64, I64, I64, I64, P, P, ctypes.c_float, P, P, P, P]),
            "b2q_rows_to_heads_f32": (I, [P, I64, I64, I64, I64, I, I64, P, P, P]),
            "b2q_attention_f32": (I, [P, P, P, I64, I64, I64, I64, I64, P, P, I64, ctypes.c_float, P, I64, P]),
            "b2q_attention_f16": (I, [P, P, P, I64, I64, I64, I64, I64, P, P, I64, ctypes.c_float, P, I64, P]),
            "b2q_attention_f16_q8": (I, [P, P, P, I64, I64, I64, I64, I64, P, P, I64, ctypes.c_float, I, P, SZ, P]),
            "b2q_layer_norm_q8": (I, [P, I64, I64, I64, ctypes.c_float, P, P, I, P, SZ, P]),
            "b2q_mul_mat_prepared_gate_residual": (I, [P, I64, I64, P, I64, P, P, P, I64, P, I64, P]),
            "b2q_norm_modulate": (I, [P, I64, I64, I64, ctypes.c_float, P, P, P, I64, P]),
            "b2q_norm_modulate_q8": (I, [P, I64, I64, I64, ctypes.c_float, P, P, I, P, SZ, P]),
            "b2q_mul_mat_prepared_peers": (I, [P, I64, I64, P, I64, P, ctypes.POINTER(ctypes.c_void_p), I, I64,
                                               I64, P]),
            "b2q_mul_mat_prepared_gelu_q8_peers": (I, [P, I64, I64, P, I64, P, ctypes.POINTER(ctypes.c_void_p), I,
                                                       I64, I64, SZ, I, P]),
            "b2q_dequantize": (I, [I, P, I64, I64, I64, I, P, I64, P]),
            "b2q_mul_mat_f32": (I, [P, I64, I64, I64, P, I64, I64, P, P, I64, P]),
            "b2q_block_dots": (I, [I, P, I64, I64, I64, P, I64, I64, P, P, SZ, P]),
            "b2q_block_dots_workspace_size": (SZ, [I64, I64, I64]),
            "b2q_mul_mat_q_simt": (I, [I, P, I64, I64, I64, P, I64, I64, P, I64, P]),
            "b2q_device_status": (I, [ctypes.POINTER(ctypes.c_uint), I]),
            "b2q_selftest_stalled_mul_mat": (I, [P, I64, I64, P, I64, P, I64, P]),
            "b2q_sparse_conv_f16_workspace_bytes": (SZ, [I64, I64, I64]),
            "b2q_sparse_conv_f16": (I, [P, I64, I64, P, I64, P, P, P, P, SZ, P]),
            "b2q_sparse_scatter_mean_workspace_bytes": (SZ, [I64, I64]),
            "b2q_sparse_scatter_mean_f16": (I, [P, I64, I64, P, P, I64, P, P, SZ, P]),
            "b2q_sparse_scatter_plan": (I, [P, I64, I64, P, SZ, P]),
            "b2q_sparse_conv_plan_bytes": (SZ, [I64]),
            "b2q_sparse_conv_plan": (I, [P, I64, P, SZ, P]),
            "b2q_sparse_conv_f16_planned_workspace_bytes": (SZ, [I64, I64, I64]),
            "b2q_sparse_conv_f16_planned": (I, [P, I64, I64, P, I64, P, P, P, P, SZ, P]),
            "b2q_sparse_scatter_mean_f16_planned": (I, [P, I64, I64, P, P, I64, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def lib():
    return _lib_obj()


def header_functions() -> list[str]:
    """Names of every function include/b2q.h declares."""
    text = open(HEADER).read()
    return re.findall(r"^B2Q_API\s+[\w\s\*]+?\b(b2q_\w+)\s*\(", text, flags=re.M)


def _check(fn: str, rc: int) -> None:
    if rc != OK:
        raise B2QError(fn, rc)


# ----------------------------------------------------------------- torch glue
def _torch():
    import torch
    return torch


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _empty_aligned(nbytes: int, device) -> "object":
    """uint8 device buffer whose data_ptr is 256-byte aligned (caching allocator
    blocks are 512-byte aligned; checked anyway)."""
    torch = _torch()
    buf = torch.empty(max(nbytes, 1) + 256, dtype=torch.uint8, device=device)
    off = (-buf.data_ptr()) % 256
    return buf[off:off + max(nbytes, 1)]


def row_bytes(wtype: int, k: int) -> int:
    if wtype == TYPE_Q4_K:
        return k // QK_K * 144
    return k // QK * BLOCK_BYTES[wtype]


def weight_packed_bytes(wtype: int, n: int, k: int) -> int:
    return lib().b2q_weight_packed_bytes(wtype, n, k)


def act_prepared_bytes(variant: int, m: int, k: int) -> int:
    return lib().b2q_act_prepared_bytes(variant, m, k)


def quantize_q8_0(x, variant: int = ACT_X86, out=None, stream=None):
    """fp32 [M, K] device tensor -> ggml block_q8_0 rows, uint8 [M, K/32*34]."""
    torch = _torch()
    assert x.dtype == torch.float32 and x.dim() == 2
    m, k = x.shape
    if out is None:
        out = torch.empty((m, row_bytes(TYPE_Q8_0, k)), dtype=torch.uint8, device=x.device)
    rc = lib().b2q_quantize_q8_0(_ptr(x), m, k, x.stride(0) * 4, _ptr(out), out.stride(0),
                                 variant, _stream(stream))
    _check("b2q_quantize_q8_0", rc)
    return out


def weight_packed_size(n: int, k: int) -> int:
    return lib().b2q_weight_packed_size(n, k)


def weight_pack(wtype: int, w, k: int, stream=None):
    """Raw ggml weight blocks uint8 [N, row_bytes] -> packed device buffer."""
    n = w.shape[0]
    size = weight_packed_bytes(wtype, n, k)
    packed = _empty_aligned(size, w.device)
    rc = lib().b2q_weight_pack(wtype, _ptr(w), n, k, w.stride(0), _ptr(packed), size, _stream(stream))
    _check("b2q_weight_pack", rc)
    return packed


def weight_pack_q4_0(w, k: int, stream=None):
    """GGUF Q4_0 rows uint8 [N, >=K/32*18] (device) -> the compact Q4_0 layout
    (GGUF footprint; the GEMM widens the nibbles on chip)."""
    n = w.shape[0]
    size = lib().b2q_weight_packed_q4_0_bytes(n, k)
    packed = _empty_aligned(size, w.device)
    rc = lib().b2q_weight_pack_q4_0(_ptr(w), n, k, w.stride(0), _ptr(packed), size, _stream(stream))
    _check("b2q_weight_pack_q4_0", rc)
    return packed


def mul_mat_prepared_q4_0(packed, n: int, k: int, act, m: int, bias=None, gate=None, resid=None, out=None,
                          stream=None):
    """Compact Q4_0 weight x prepared Q8_0 activations -> fp32 [m, n]; with
    resid: resid + gate * (w.act + bias) (out=resid updates in place)."""
    torch = _torch()
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=act.device)
    rc = lib().b2q_mul_mat_prepared_q4_0(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), _ptr(gate), _ptr(resid),
                                         resid.stride(0) * 4 if resid is not None else 0, _ptr(out),
                                         out.stride(0) * 4, _stream(stream))
    _check("b2q_mul_mat_prepared_q4_0", rc)
    return out


def mul_mat_prepared_q4_0_gelu_q8(packed, n: int, k: int, act, m: int, bias=None, variant: int = ACT_X86,
                                  out=None, stream=None):
    size = act_prepared_size(m, n)
    if out is None:
        out = _empty_aligned(size, act.device)
    rc = lib().b2q_mul_mat_prepared_q4_0_gelu_q8(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), _ptr(out),
                                                 out.numel() * out.element_size(), variant, _stream(stream))
    _check("b2q_mul_mat_prepared_q4_0_gelu_q8", rc)
    return out


def weight_upload(wtype: int, host_w, k: int, staging_bytes: int = 8 << 20, device=None, stream=None):
    """Raw ggml weight blocks in host memory (numpy uint8 [N, >=row_bytes]) ->
    packed device buffer, through a staging buffer of staging_bytes."""
    import numpy as np
    torch = _torch()
    host_w = np.asarray(host_w)
    n = host_w.shape[0]
    dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    size = weight_packed_bytes(wtype, n, k)
    packed = _empty_aligned(size, dev)
    staging = _empty_aligned(staging_bytes, dev)
    rc = lib().b2q_weight_upload(wtype, host_w.ctypes.data, n, k, host_w.strides[0], _ptr(staging), staging_bytes,
                                 _ptr(packed), size, _stream(stream))
    _check("b2q_weight_upload", rc)
    torch.cuda.current_stream(dev).synchronize() if stream is None else stream.synchronize()
    return packed


def workspace_size(m: int, n: int, k: int, packed_weight: bool) -> int:
    return lib().b2q_mul_mat_workspace_size(m, n, k, 1 if packed_weight else 0)


def workspace(m: int, n: int, k: int, packed_weight: bool, device):
    return _empty_aligned(workspace_size(m, n, k, packed_weight), device)


def mul_mat(wtype: int, w, x, k: int | None = None, bias=None, variant: int | None = None,
            out=None, ws=None, stream=None):
    """ggml_mul_mat(w, x) (+ bias): w raw blocks uint8 [N, >=row_bytes] (TYPE_F16:
    float16 [N, >=K]), x fp32 [M, K] -> [M, N].  variant defaults to ACT_X86
    (ACT_Q8_K for Q4_K weights)."""
    torch = _torch()
    m, kk = x.shape
    k = kk if k is None else k
    n = w.shape[0]
    if variant is None:
        variant = ACT_Q8_K if wtype == TYPE_Q4_K else ACT_X86
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    if ws is None:
        ws = _empty_aligned(lib().b2q_mul_mat_workspace_bytes(wtype, m, n, k, 0), x.device)
    rc = lib().b2q_mul_mat(wtype, _ptr(w), w.stride(0) * w.element_size(), n, k, _ptr(x), m, x.stride(0) * 4,
                           _ptr(bias), _ptr(out), out.stride(0) * 4, variant, _ptr(ws), ws.numel(),
                           _stream(stream))
    _check("b2q_mul_mat", rc)
    return out


def mul_mat_packed(packed, n: int, k: int, x, bias=None, variant: int = ACT_X86, out=None,
                   ws=None, stream=None):
    torch = _torch()
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    if ws is None:
        wt = TYPE_Q4_K if variant == ACT_Q8_K else TYPE_Q8_0
        ws = _empty_aligned(lib().b2q_mul_mat_workspace_bytes(wt, m, n, k, 1), x.device)
    rc = lib().b2q_mul_mat_packed(_ptr(packed), n, k, _ptr(x), m, x.stride(0) * 4, _ptr(bias),
                                  _ptr(out), out.stride(0) * 4, variant, _ptr(ws), ws.numel(),
                                  _stream(stream))
    _check("b2q_mul_mat_packed", rc)
    return out


NOALLOC_SCRATCH_BYTES = 32 << 20  # B2Q_NOALLOC_SCRATCH_BYTES


def mul_mat_packed_noalloc(packed, n: int, k: int, x, bias=None, variant: int = ACT_X86, out=None,
                           stream=None):
    """mul_mat_packed with the activations in the library's fixed device array
    (no workspace); calls on one device must not overlap."""
    torch = _torch()
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    rc = lib().b2q_mul_mat_packed_noalloc(_ptr(packed), n, k, _ptr(x), m, x.stride(0) * 4,
                                          _ptr(bias), _ptr(out), out.stride(0) * 4, variant,
                                          _stream(stream))
    _check("b2q_mul_mat_packed_noalloc", rc)
    return out


def mul_mat_prepared_peers(packed, n: int, k: int, act, m: int, y_peers, y_col0: int,
                           y_row_stride_bytes: int, bias=None, stream=None):
    """Column-parallel mul_mat: this rank's weight rows [y_col0, y_col0 + n)
    written into every buffer of y_peers (a list of device addresses)."""
    arr = (ctypes.c_void_p * len(y_peers))(*[int(p) for p in y_peers])
    rc = lib().b2q_mul_mat_prepared_peers(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), arr, len(y_peers),
                                          y_col0, y_row_stride_bytes, _stream(stream))
    _check("b2q_mul_mat_prepared_peers", rc)


def mul_mat_prepared_gelu_q8_peers(packed, n: int, k: int, act, m: int, act_peers, n_total: int, col0: int,
                                   act_bytes: int, bias=None, variant: int = ACT_X86, stream=None):
    """Column-parallel GELU + Q8_0: this rank's weight rows [col0, col0 + n)
    quantized straight into every prepared-activation buffer of act_peers (a
    list of device addresses, each laid out for [m, n_total])."""
    arr = (ctypes.c_void_p * len(act_peers))(*[int(p) for p in act_peers])
    rc = lib().b2q_mul_mat_prepared_gelu_q8_peers(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), arr,
                                                  len(act_peers), n_total, col0, act_bytes, variant,
                                                  _stream(stream))
    _check("b2q_mul_mat_prepared_gelu_q8_peers", rc)


def dequantize(wtype: int, w, k: int, out_type: int = TYPE_F32, out=None, stream=None):
    """GGUF rows uint8 [N, >= row bytes] (device) -> fp32 (or fp16) [N, k]:
    the reference's as_f32 / as_f16 cast of a quantized weight."""
    torch = _torch()
    n = w.shape[0]
    dt = torch.float32 if out_type == TYPE_F32 else torch.float16
    if out is None:
        out = torch.empty((n, k), dtype=dt, device=w.device)
    rc = lib().b2q_dequantize(wtype, _ptr(w), w.stride(0), n, k, out_type, _ptr(out),
                              out.stride(0) * out.element_size(), _stream(stream))
    _check("b2q_dequantize", rc)
    return out


def mul_mat_f32(w, x, bias=None, out=None, stream=None):
    """Strict F32 mul_mat: fp32 w [N, K] (the as_f32 weight) x fp32 x [M, K]
    -> fp32 [M, N] (+ bias), every product and sum in fp32."""
    torch = _torch()
    n, k = w.shape
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    rc = lib().b2q_mul_mat_f32(_ptr(w), w.stride(0) * 4, n, k, _ptr(x), x.stride(0) * 4, m, _ptr(bias), _ptr(out),
                               out.stride(0) * 4, _stream(stream))
    _check("b2q_mul_mat_f32", rc)
    return out


def act_prepared_size(m: int, k: int) -> int:
    return lib().b2q_act_prepared_size(m, k)


def act_prepare(x, variant: int = ACT_X86, out=None, stream=None):
    """fp32 [M, K] -> prepared Q8_0 (or, with ACT_Q8_K, Q8_K) activations
    (device buffer in the GEMM's layout)."""
    m, k = x.shape
    size = act_prepared_bytes(variant, m, k)
    if out is None:
        out = _empty_aligned(size, x.device)
    rc = lib().b2q_act_prepare(_ptr(x), m, k, x.stride(0) * 4, variant, _ptr(out), out.numel(),
                               _stream(stream))
    _check("b2q_act_prepare", rc)
    return out


def mul_mat_prepared(packed, n: int, k: int, act, m: int, bias=None, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=act.device)
    rc = lib().b2q_mul_mat_prepared(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), _ptr(out),
                                    out.stride(0) * 4, _stream(stream))
    _check("b2q_mul_mat_prepared", rc)
    return out


def mul_mat_prepared_gelu_q8(packed, n: int, k: int, act, m: int, bias=None,
                             variant: int = ACT_X86, out=None, stream=None):
    """fc1 with bias + GELU + Q8_0 quantize fused: returns the prepared
    activations of the next mul_mat (m rows, k_next = n) instead of fp32 y."""
    size = act_prepared_size(m, n)
    if out is None:
        out = _empty_aligned(size, act.device)
    rc = lib().b2q_mul_mat_prepared_gelu_q8(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), _ptr(out),
                                            out.numel() * out.element_size(), variant,
                                            _stream(stream))
    _check("b2q_mul_mat_prepared_gelu_q8", rc)
    return out


def mul_mat_prepared_gate_residual(packed, n: int, k: int, act, m: int, resid, bias=None, gate=None,
                                   out=None, stream=None):
    """resid + gate * (mul_mat + bias), fp32 [m, n]; out=resid updates the residual in place."""
    torch = _torch()
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=act.device)
    rc = lib().b2q_mul_mat_prepared_gate_residual(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), _ptr(gate),
                                                  _ptr(resid), resid.stride(0) * 4, _ptr(out),
                                                  out.stride(0) * 4, _stream(stream))
    _check("b2q_mul_mat_prepared_gate_residual", rc)
    return out


def mul_mat_prepared_q4_k(packed, n: int, k: int, act, m: int, bias=None, gate=None, resid=None, out=None,
                          stream=None):
    """Q4_K packed weight x prepared Q8_K activations -> fp32 [m, n]; with
    resid: resid + gate * (w.x + bias) (out=resid updates it in place)."""
    torch = _torch()
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=act.device)
    rc = lib().b2q_mul_mat_prepared_q4_k(_ptr(packed), n, k, _ptr(act), m, _ptr(bias), _ptr(gate), _ptr(resid),
                                         resid.stride(0) * 4 if resid is not None else 0, _ptr(out),
                                         out.stride(0) * 4, _stream(stream))
    _check("b2q_mul_mat_prepared_q4_k", rc)
    return out


def qkv_heads(qkv, B: int, T: int, H: int, D: int, gamma_q=None, gamma_k=None, eps: float = 1e-6, stream=None):
    """fused qkv rows fp32 [B*T, 3*H*D] -> (q, k, v) fp16 [B, H, T, D] (q, k RMS-normed per head)."""
    torch = _torch()
    q, k, v = (torch.empty((B, H, T, D), dtype=torch.float16, device=qkv.device) for _ in range(3))
    rc = lib().b2q_qkv_heads(_ptr(qkv), B, T, H, D, qkv.stride(0) * 4, _ptr(gamma_q), _ptr(gamma_k), eps,
                             _ptr(q), _ptr(k), _ptr(v), _stream(stream))
    _check("b2q_qkv_heads", rc)
    return q, k, v


def rows_to_heads(src, B: int, T: int, H: int, D: int, parts: int = 1, stream=None):
    """fp32 rows [B*T, parts*H*D] -> parts fp16 tensors [B, H, T, D] (no norm)."""
    torch = _torch()
    outs = [torch.empty((B, H, T, D), dtype=torch.float16, device=src.device) for _ in range(parts)]
    rc = lib().b2q_rows_to_heads(_ptr(src), B, T, H, D, parts, src.stride(0) * 4, _ptr(outs[0]),
                                 _ptr(outs[1]) if parts == 2 else None, _stream(stream))
    _check("b2q_rows_to_heads", rc)
    return outs


def mul_mat_prepared_heads(packed, n: int, k: int, act, B: int, T: int, H: int, D: int = 64, bias=None,
                           stream=None):
    """mul_mat_prepared (+ bias) straight into fp16 attention heads: n = parts*H*D
    output columns -> parts tensors [B, H, T, D], the bytes of mul_mat_prepared
    followed by rows_to_heads.  Tensor-core path only (B*T > 8, D = 64)."""
    torch = _torch()
    parts = n // (H * D)
    outs = [torch.empty((B, H, T, D), dtype=torch.float16, device=act.device) for _ in range(parts)]
    rc = lib().b2q_mul_mat_prepared_heads_f16(_ptr(packed), n, k, _ptr(act), B * T, _ptr(bias), B, T, H, D, parts,
                                              _ptr(outs[0]), _ptr(outs[1]) if parts == 2 else None,
                                              _stream(stream))
    _check("b2q_mul_mat_prepared_heads_f16", rc)
    return outs


def qkv_heads_f32(qkv, B: int, T: int, H: int, D: int, gamma_q=None, gamma_k=None, eps: float = 1e-6,
                  stream=None):
    """qkv_heads with fp32 outputs [B, H, T, D] (the F32 attention contract)."""
    torch = _torch()
    q, k, v = (torch.empty((B, H, T, D), dtype=torch.float32, device=qkv.device) for _ in range(3))
    rc = lib().b2q_qkv_heads_f32(_ptr(qkv), B, T, H, D, qkv.stride(0) * 4, _ptr(gamma_q), _ptr(gamma_k), eps,
                                 _ptr(q), _ptr(k), _ptr(v), _stream(stream))
    _check("b2q_qkv_heads_f32", rc)
    return q, k, v


def rows_to_heads_f32(src, B: int, T: int, H: int, D: int, parts: int = 1, stream=None):
    """rows_to_heads with fp32 outputs [B, H, T, D]."""
    torch = _torch()
    outs = [torch.empty((B, H, T, D), dtype=torch.float32, device=src.device) for _ in range(parts)]
    rc = lib().b2q_rows_to_heads_f32(_ptr(src), B, T, H, D, parts, src.stride(0) * 4, _ptr(outs[0]),
                                     _ptr(outs[1]) if parts == 2 else None, _stream(stream))
    _check("b2q_rows_to_heads_f32", rc)
    return outs


def attention_f32(q, k, v, k2=None, v2=None, scale: float | None = None, out=None, stream=None):
    """F32-contract attention: q [B, H, Tq, D], k, v [B, H, Tk, D] fp32 (plus an
    optional second key source k2, v2 [B, H, Tk2, D]) -> fp32 rows [B*Tq, H*D]."""
    import math
    torch = _torch()
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    Tk2 = k2.shape[2] if k2 is not None else 0
    for t in (q, k, v, k2, v2):
        assert t is None or (t.dtype == torch.float32 and t.is_contiguous())
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B * Tq, H * D), dtype=torch.float32, device=q.device)
    rc = lib().b2q_attention_f32(_ptr(q), _ptr(k), _ptr(v), B, H, Tq, Tk, D, _ptr(k2), _ptr(v2), Tk2, scale,
                                 _ptr(out), out.stride(0) * 4, _stream(stream))
    _check("b2q_attention_f32", rc)
    return out


def attention_f16(q, k, v, k2=None, v2=None, scale: float | None = None, out=None, stream=None):
    """Tensor-core attention (D = 64): q [B, H, Tq, 64], k, v [B, H, Tk, 64] fp16
    (plus an optional second key source k2, v2) -> fp16 rows [B*Tq, H*64]."""
    import math
    torch = _torch()
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    Tk2 = k2.shape[2] if k2 is not None else 0
    for t in (q, k, v, k2, v2):
        assert t is None or (t.dtype == torch.float16 and t.is_contiguous())
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty((B * Tq, H * D), dtype=torch.float16, device=q.device)
    rc = lib().b2q_attention_f16(_ptr(q), _ptr(k), _ptr(v), B, H, Tq, Tk, D, _ptr(k2), _ptr(v2), Tk2, scale,
                                 _ptr(out), out.stride(0) * 2, _stream(stream))
    _check("b2q_attention_f16", rc)
    return out


def attention_f16_q8(q, k, v, k2=None, v2=None, scale: float | None = None, variant: int = ACT_X86, out=None,
                     stream=None):
    """attention_f16 with the output as the output projection's Q8_0 prepared
    activations (rows b*Tq + t, K = H*64): the bytes of heads_act_prepare of
    attention_f16's output, in one launch."""
    import math
    torch = _torch()
    B, H, Tq, D = q.shape
    Tk = k.shape[2]
    Tk2 = k2.shape[2] if k2 is not None else 0
    for t in (q, k, v, k2, v2):
        assert t is None or (t.dtype == torch.float16 and t.is_contiguous())
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    size = act_prepared_size(B * Tq, H * D)
    if out is None:
        out = _empty_aligned(size, q.device)
    rc = lib().b2q_attention_f16_q8(_ptr(q), _ptr(k), _ptr(v), B, H, Tq, Tk, D, _ptr(k2), _ptr(v2), Tk2, scale,
                                    variant, _ptr(out), out.numel(), _stream(stream))
    _check("b2q_attention_f16_q8", rc)
    return out


def layer_norm_q8(x, eps: float = 1e-6, weight=None, bias=None, variant: int = ACT_X86, out=None, stream=None):
    """gb_layer_norm (affine weight, bias) straight into Q8_0 prepared activations."""
    m, c = x.shape
    size = act_prepared_size(m, c)
    if out is None:
        out = _empty_aligned(size, x.device)
    rc = lib().b2q_layer_norm_q8(_ptr(x), m, c, x.stride(0) * 4, eps, _ptr(weight), _ptr(bias), variant, _ptr(out),
                                 out.numel(), _stream(stream))
    _check("b2q_layer_norm_q8", rc)
    return out


def sparse_conv_f16(x16, w16, bias16, indices, out=None, ws=None, stream=None):
    """F16 submanifold convolution: x16 [tokens, C] fp16, w16 [Cout, 27*C] fp16,
    bias16 [Cout] fp16 or None, indices int32 [27, tokens] (offset-major, -1 =
    missing) -> fp16 [tokens, Cout]."""
    torch = _torch()
    tokens, C = x16.shape
    cout = w16.shape[0]
    assert w16.shape[1] == 27 * C and indices.shape == (27, tokens)
    if out is None:
        out = torch.empty((tokens, cout), dtype=torch.float16, device=x16.device)
    if ws is None:
        ws = _empty_aligned(max(lib().b2q_sparse_conv_f16_workspace_bytes(tokens, C, cout), 256), x16.device)
    rc = lib().b2q_sparse_conv_f16(_ptr(x16), tokens, C, _ptr(w16), cout, _ptr(bias16), _ptr(indices), _ptr(out),
                                   _ptr(ws), ws.numel(), _stream(stream))
    _check("b2q_sparse_conv_f16", rc)
    return out


def sparse_scatter_mean_f16(x16, rows, counts, coarse: int, out=None, ws=None, stream=None):
    """F16 scatter-mean: x16 [fine, C] fp16, rows int32 [fine] (target coarse
    row), counts fp32 [coarse] (divisors) -> fp16 [coarse, C]."""
    torch = _torch()
    fine, C = x16.shape
    if out is None:
        out = torch.empty((coarse, C), dtype=torch.float16, device=x16.device)
    if ws is None:
        ws = _empty_aligned(max(lib().b2q_sparse_scatter_mean_workspace_bytes(fine, coarse), 256), x16.device)
    rc = lib().b2q_sparse_scatter_mean_f16(_ptr(x16), fine, C, _ptr(rows), _ptr(counts), coarse, _ptr(out),
                                           _ptr(ws), ws.numel(), _stream(stream))
    _check("b2q_sparse_scatter_mean_f16", rc)
    return out


def sparse_conv_plan(indices, stream=None):
    """Occupied (token, neighbour) pairs of a 27-neighbour table int32 [27, tokens],
    for sparse_conv_f16_planned (reusable while the table does not change)."""
    tokens = indices.shape[1]
    plan = _empty_aligned(lib().b2q_sparse_conv_plan_bytes(tokens), indices.device)
    rc = lib().b2q_sparse_conv_plan(_ptr(indices), tokens, _ptr(plan), plan.numel(), _stream(stream))
    _check("b2q_sparse_conv_plan", rc)
    return plan


def sparse_conv_f16_planned(x16, w16, bias16, plan, out=None, ws=None, stream=None):
    """sparse_conv_f16 over the occupied pairs of a plan (C % 64 == 0, Cout % 8 == 0)."""
    torch = _torch()
    tokens, C = x16.shape
    cout = w16.shape[0]
    if out is None:
        out = torch.empty((tokens, cout), dtype=torch.float16, device=x16.device)
    if ws is None:
        ws = _empty_aligned(max(lib().b2q_sparse_conv_f16_planned_workspace_bytes(tokens, C, cout), 256), x16.device)
    rc = lib().b2q_sparse_conv_f16_planned(_ptr(x16), tokens, C, _ptr(w16), cout, _ptr(bias16), _ptr(plan), _ptr(out),
                                           _ptr(ws), ws.numel(), _stream(stream))
    _check("b2q_sparse_conv_f16_planned", rc)
    return out


def sparse_scatter_plan(rows, coarse: int, stream=None):
    """Child lists of every coarse row for sparse_scatter_mean_f16_planned
    (reusable while rows does not change)."""
    fine = rows.shape[0]
    plan = _empty_aligned(max(lib().b2q_sparse_scatter_mean_workspace_bytes(fine, coarse), 256), rows.device)
    rc = lib().b2q_sparse_scatter_plan(_ptr(rows), fine, coarse, _ptr(plan), plan.numel(), _stream(stream))
    _check("b2q_sparse_scatter_plan", rc)
    return plan


def sparse_scatter_mean_f16_planned(x16, plan, counts, coarse: int, out=None, stream=None):
    torch = _torch()
    fine, C = x16.shape
    if out is None:
        out = torch.empty((coarse, C), dtype=torch.float16, device=x16.device)
    rc = lib().b2q_sparse_scatter_mean_f16_planned(_ptr(x16), fine, C, _ptr(plan), _ptr(counts), coarse, _ptr(out),
                                                   _stream(stream))
    _check("b2q_sparse_scatter_mean_f16_planned", rc)
    return out


def heads_act_prepare(o, variant: int = ACT_X86, out=None, stream=None):
    """attention output fp16 [B, H, T, D] (any strides, d contiguous) -> Q8_0
    prepared activations for rows (b, t), K = H*D."""
    B, H, T, D = o.shape
    assert o.stride(3) == 1
    size = act_prepared_size(B * T, H * D)
    if out is None:
        out = _empty_aligned(size, o.device)
    rc = lib().b2q_heads_act_prepare(_ptr(o), B, T, H, D, o.stride(0), o.stride(1), o.stride(2), variant,
                                     _ptr(out), out.numel(), _stream(stream))
    _check("b2q_heads_act_prepare", rc)
    return out


def gelu(x, out=None, stream=None):
    """ggml_gelu (CPU-backend arithmetic) on an fp32 [rows, cols] CUDA tensor."""
    torch = _torch()
    rows, cols = x.shape
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.float32, device=x.device)
    rc = lib().b2q_gelu(_ptr(x), rows, cols, x.stride(0) * 4, _ptr(out), out.stride(0) * 4,
                        _stream(stream))
    _check("b2q_gelu", rc)
    return out


def norm_modulate(x, eps: float = 1e-6, scale=None, shift=None, out=None, stream=None):
    """ggml_norm + adaLN modulate, fp32 [M, C] -> fp32 [M, C] (CUDA tensors)."""
    torch = _torch()
    m, c = x.shape
    if out is None:
        out = torch.empty((m, c), dtype=torch.float32, device=x.device)
    rc = lib().b2q_norm_modulate(_ptr(x), m, c, x.stride(0) * 4, eps, _ptr(scale), _ptr(shift), _ptr(out),
                                 out.stride(0) * 4, _stream(stream))
    _check("b2q_norm_modulate", rc)
    return out


def norm_modulate_q8(x, eps: float = 1e-6, scale=None, shift=None, variant: int = ACT_X86, out=None,
                     stream=None):
    """ggml_norm + adaLN modulate straight into the next mul_mat's prepared Q8_0 activations."""
    m, c = x.shape
    size = act_prepared_size(m, c)
    if out is None:
        out = _empty_aligned(size, x.device)
    rc = lib().b2q_norm_modulate_q8(_ptr(x), m, c, x.stride(0) * 4, eps, _ptr(scale), _ptr(shift), variant,
                                    _ptr(out), out.numel() * out.element_size(), _stream(stream))
    _check("b2q_norm_modulate_q8", rc)
    return out


def block_dots(wtype: int, w, a, k: int, stream=None):
    """int32 [M, N, K/32] block dots from the tensor-core kernel (a: Q8_0 blocks [M, .])."""
    torch = _torch()
    n, m = w.shape[0], a.shape[0]
    dots = torch.empty((m, n, k // QK), dtype=torch.int32, device=w.device)
    ws = _empty_aligned(lib().b2q_block_dots_workspace_size(m, n, k), w.device)
    rc = lib().b2q_block_dots(wtype, _ptr(w), w.stride(0), n, k, _ptr(a), m, a.stride(0),
                              _ptr(dots), _ptr(ws), ws.numel(), _stream(stream))
    _check("b2q_block_dots", rc)
    return dots


def mul_mat_q_simt(wtype: int, w, a, k: int, stream=None):
    """CUDA-core check kernel, ggml x86 accumulation order: y [M, N] fp32."""
    torch = _torch()
    n, m = w.shape[0], a.shape[0]
    y = torch.empty((m, n), dtype=torch.float32, device=w.device)
    rc = lib().b2q_mul_mat_q_simt(wtype, _ptr(w), w.stride(0), n, k, _ptr(a), m, a.stride(0),
                                  _ptr(y), y.stride(0) * 4, _stream(stream))
    _check("b2q_mul_mat_q_simt", rc)
    return y


def device_status(clear: bool = True) -> int:
    code = ctypes.c_uint(0)
    rc = lib().b2q_device_status(ctypes.byref(code), 1 if clear else 0)
    if rc not in (OK, 6):
        raise B2QError("b2q_device_status", rc)
    return code.value
