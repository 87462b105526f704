"""Shared test helpers: the reference test's input generator and pass criteria,
seeded synthetic cases, error metrics."""
from __future__ import annotations

import numpy as np

import oracle as O


def sample(index: np.ndarray, salt: int) -> np.ndarray:
    """Stateless hash generator of the reference's matmul regression test
    (cpp_ggml/src/matmul_backend_test.cpp:17-22): values in {-128..128}/128.
    Kept value-identical so the same inputs drive both tests."""
    idx = np.asarray(index, dtype=np.uint64)
    v = (idx * np.uint64(747796405) + np.uint64(salt) * np.uint64(2891336453)) & np.uint64(0xFFFFFFFF)
    v = ((((v >> ((v >> np.uint64(28)) + np.uint64(4))) ^ v) * np.uint64(277803737))
         & np.uint64(0xFFFFFFFF))
    v = (v >> np.uint64(22)) ^ v
    return ((v % np.uint64(257)).astype(np.int64) - 128).astype(np.float32) / np.float32(128.0)


def reference_check(actual: np.ndarray, w_deq: np.ndarray, x: np.ndarray, iteration: int,
                    probes: int = 1024) -> dict:
    """Pass criteria of cpp_ggml/src/matmul_backend_test.cpp:68-89: all outputs
    finite; at 1024 probe points the fp64 dot of the dequantized weights with the
    fp32 inputs must correlate >= 0.9999 with the output.

    The reference's fixed max-abs bound (0.05) presumes unquantized activations
    (its GPU backends dequantize in the shader; on the CPU backend the input type
    must equal the weight type, :171-181, so Q8_0 was never run there).  ggml's
    CPU path quantizes every activation block to Q8_0, whose per-value error is
    at most d/2 plus the fp16 rounding of d (< 0.07 d), so each probe is checked
    against its own rigorous bound  sum_k |w_deq[k]| * 0.57 * d_block(k)  + 1e-5."""
    M, N = actual.shape
    K = x.shape[1]
    flat = actual.reshape(-1)
    nonfinite = int(np.sum(~np.isfinite(flat)))
    offs = np.array([flat.size - 1 if p == 0 else (p * 104729 + iteration * 37) % flat.size
                     for p in range(probes)], dtype=np.int64)
    rows, cols = offs // N, offs % N
    expected = np.einsum("pk,pk->p", w_deq[cols].astype(np.float64), x[rows].astype(np.float64))
    got = flat[offs].astype(np.float64)
    err = np.abs(got - expected)
    d = np.abs(x.reshape(M, K // 32, 32)).max(axis=2).astype(np.float64) / 127.0   # [M, K/32]
    bound = np.einsum("pbi,pb->p", np.abs(w_deq[cols].reshape(-1, K // 32, 32)).astype(np.float64),
                      0.57 * d[rows]) + 1e-5
    corr = np.corrcoef(expected, got)[0, 1] if np.std(expected) > 0 and np.std(got) > 0 else 0.0
    ok = nonfinite == 0 and np.isfinite(corr) and corr >= 0.9999 and bool(np.all(err <= bound))
    return {"ok": bool(ok), "nonfinite": nonfinite, "mae": float(err.mean()),
            "max": float(err.max()), "max_over_bound": float(np.max(err / bound)),
            "corr": float(corr)}


def rel_frobenius(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def make_case(seed: int, M: int, N: int, K: int, wtype: int, w_std: float = 0.02,
              gelu: bool = False):
    """Seeded synthetic case: W ~ N(0, w_std) quantized with the ggml reference
    quantizer, X ~ N(0, 1) (or GELU-tanh of it, the fc2 input)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * w_std).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    if gelu:
        x = gelu_tanh(x)
    wq = O.quantize(w, wtype)
    return w, wq, x


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    x64 = x.astype(np.float64)
    return (0.5 * x64 * (1.0 + np.tanh(0.7978845608028654 * (x64 + 0.044715 * x64 ** 3)))).astype(np.float32)
