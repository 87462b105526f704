"""Generate tests/golden/q_golden.npz -- golden vectors for the Q8_0 / Q4_0 path.

Independent of this repository's oracle: block bytes come from gguf-py 0.19.0
(``gguf.quants``, whose Q8_0 / Q4_0 quantizers are documented there as
bit-exact with ggml's reference quantizers; the reference converter uses the
same package, cpp_ggml/scripts/gguf_schema.py:11-52), and the expected int32
block dots and fp64 products are computed here with plain numpy from those
bytes.  Run in a container where gguf-py is importable:

    python tests/golden/make_golden.py

Shapes follow the reference's matmul regression test: K = 256, N = 65 output
rows, M = 33 tokens (the tail-tile shape of cpp_ggml/src/matmul_backend_test.cpp:182).
Weights ~ N(0, 0.02), activations ~ N(0, 1), plus planted edge blocks (all
zero, tiny, huge, exact rounding ties).
"""
from __future__ import annotations

import importlib.metadata
import os

import numpy as np
from gguf import GGMLQuantizationType as T
import gguf.quants as gq

HERE = os.path.dirname(os.path.abspath(__file__))
K, N, M = 256, 65, 33


def codes_and_scales(blocks: np.ndarray, qtype) -> tuple[np.ndarray, np.ndarray]:
    """uint8 rows of ggml blocks -> (int codes [rows, K], fp32 scales [rows, K/32])."""
    rows = blocks.shape[0]
    bpb = 34 if qtype == T.Q8_0 else 18
    b = blocks.reshape(rows, -1, bpb)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float32)[:, :, 0]
    if qtype == T.Q8_0:
        q = b[:, :, 2:].view(np.int8).astype(np.int32)
    else:
        lo = (b[:, :, 2:] & 0x0F).astype(np.int32) - 8
        hi = (b[:, :, 2:] >> 4).astype(np.int32) - 8
        q = np.concatenate([lo, hi], axis=2)
    return q.reshape(rows, -1), d


def main() -> None:
    rng = np.random.default_rng(20261201)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    # planted edge blocks
    w[0, 0:32] = 0.0                       # all-zero block -> d = 0, codes 0
    w[1, 32:64] = 1e-7                     # tiny values (fp16-subnormal scale)
    w[2, 64:96] = np.linspace(-3, 3, 32)   # large spread
    x[0, 0:32] = 0.0
    x[1, 32:64] = np.arange(32, dtype=np.float32) - 15.5   # many .5 ties after scaling
    x[2, 64:96] = 1e4 * rng.standard_normal(32).astype(np.float32)
    x[3, 96:128] = -2.0                    # constant block: every code = -127

    out = {"K": np.int64(K), "N": np.int64(N), "M": np.int64(M), "w": w, "x": x,
           "gguf_version": np.array(importlib.metadata.version("gguf"))}
    a = gq.quantize(x, T.Q8_0)             # ggml reference activation quantizer
    out["a_q8_ref"] = a
    qa, da = codes_and_scales(a, T.Q8_0)
    for name, qt in (("q8_0", T.Q8_0), ("q4_0", T.Q4_0)):
        wb = gq.quantize(w, qt)
        out[f"w_{name}"] = wb
        out[f"w_{name}_dequant"] = gq.dequantize(wb, qt).astype(np.float32)
        qw, dw = codes_and_scales(wb, qt)
        # int32 block dots S_b(n, m) -> [M, N, K/32]
        dots = np.einsum("nbi,mbi->mnb", qw.reshape(N, -1, 32), qa.reshape(M, -1, 32)).astype(np.int32)
        out[f"dots_{name}"] = dots
        # fp64 reference of the exact dequantized product
        out[f"y_f64_{name}"] = (gq.dequantize(a, T.Q8_0).astype(np.float64)
                                @ gq.dequantize(wb, qt).astype(np.float64).T)
        # sum_b fp32(dw*da) * S_b in fp64 (exact form of ggml's per-block scaling)
        scale = (dw[None, :, :] * da[:, None, :]).astype(np.float32).astype(np.float64)
        out[f"y_blockscale_{name}"] = np.sum(scale * dots.astype(np.float64), axis=2)
    np.savez_compressed(os.path.join(HERE, "q_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "q_golden.npz"))


def main_q4_k() -> None:
    """q4k_golden.npz: seeded random Q4_K blocks (any bytes with finite fp16
    d / dmin are a valid weight; the quantizer runs offline) and gguf-py's
    dequantization of them -- pins the block layout and the 6-bit scale / min
    unpacking.  Includes blocks whose packed scale bytes have the high bits
    set (the j >= 4 unpacking path)."""
    rng = np.random.default_rng(4242)
    n, k = 9, 512
    nb = k // 256
    b = rng.integers(0, 256, size=(n, nb, 144), dtype=np.uint8)
    d = np.abs(rng.standard_normal((n, nb)) * 0.01).astype(np.float16)
    dm = np.abs(rng.standard_normal((n, nb)) * 0.01).astype(np.float16)
    b[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    b[:, :, 2:4] = dm.view(np.uint8).reshape(n, nb, 2)
    b[0, 0, 4:16] = 0xFF          # every scale and min at 63
    b[1, 0, 4:16] = 0x00          # every scale and min at 0
    w = b.reshape(n, nb * 144)
    out = {"w_q4_k": w, "w_q4_k_dequant": gq.dequantize(w, T.Q4_K).astype(np.float32),
           "gguf_version": np.array(importlib.metadata.version("gguf"))}
    np.savez_compressed(os.path.join(HERE, "q4k_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "q4k_golden.npz"))


if __name__ == "__main__":
    main()
    main_q4_k()
