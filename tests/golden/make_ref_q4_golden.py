"""Generate tests/golden/ref_q4_0.npz -- Q4_0 weight bytes from the reference's
own quantizer.

The reference ships a Python Q4_0 quantizer that it documents as matching
ggml's ``quantize_row_q4_0_ref`` byte for byte
(cpp_ggml/scripts/gguf_schema.py:27-52; used by its converter,
cpp_ggml/scripts/convert_sam3d_to_gguf.py).  This script imports that function
from a reference checkout (read-only) and records its output on:

- ``w_small``: the 65 x 256 N(0, 0.02) matrix of q_golden.npz, with planted
  edge blocks (all zero, +max / -max ties, tiny, huge, the exact x*id + 8.5
  boundaries, fp16-subnormal scales);
- the BASELINE weight shapes (fc1 4096 x 1024 and fc2 1024 x 4096, N(0, 0.02)
  from the seeds stored here): the first 16 rows in full and the SHA-256 of
  all bytes, so the fixture stays small.

Run where the reference is present:

    python tests/golden/make_ref_q4_golden.py [path/to/reference]
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_REF = os.path.join(os.sep, "root", "reference")
BIG = (("fc1", 4096, 1024, 101), ("fc2", 1024, 4096, 102))  # name, rows N, K, seed


def load_reference_quantizer(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "cpp_ggml", "scripts"))
    try:
        import gguf_schema  # the reference's module
    finally:
        sys.path.pop(0)
    return gguf_schema.quantize_q4_0


def small_matrix() -> np.ndarray:
    g = np.load(os.path.join(HERE, "q_golden.npz"))
    w = np.array(g["w"], dtype=np.float32)  # 65 x 256
    w[3, 0:32] = 0.0
    w[3, 5] = 0.5
    w[3, 9] = -0.5                                  # +max / -max tie: the first one sets the sign
    w[4, 32:64] = np.float32(1e-6) * np.arange(-16, 16, dtype=np.float32)  # fp16-subnormal scale
    w[5, 64:96] = np.float32(3e4) * np.sin(np.arange(32, dtype=np.float32))  # huge
    base = np.arange(32, dtype=np.float32) - 16.0   # x*id lands on k + 0.5 steps for max = -16
    w[6, 96:128] = base * np.float32(0.5)
    w[7, 128:160] = -(base * np.float32(0.25))
    w[8, 160:192] = np.float32(1.0)                 # constant block: every code = 0 (x*id = -8)
    w[9, 192:224] = np.float32(-1.0)                # constant negative block: every code = 0
    return w


def big_matrix(n: int, k: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((n, k)) * 0.02).astype(np.float32)


def main() -> None:
    ref_root = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF
    quantize_q4_0 = load_reference_quantizer(ref_root)
    out = {}
    w = small_matrix()
    out["w_small"] = w
    out["q4_small"] = quantize_q4_0(w).reshape(w.shape[0], -1)
    for name, n, k, seed in BIG:
        wb = quantize_q4_0(big_matrix(n, k, seed)).reshape(n, -1)
        out[f"{name}_shape"] = np.array([n, k, seed], dtype=np.int64)
        out[f"{name}_head"] = wb[:16]
        out[f"{name}_sha256"] = np.array(hashlib.sha256(wb.tobytes()).hexdigest())
    np.savez_compressed(os.path.join(HERE, "ref_q4_0.npz"), **out)
    print("wrote", os.path.join(HERE, "ref_q4_0.npz"))


if __name__ == "__main__":
    main()
