"""F16-weight GGML_OP_MUL_MAT (b2q_mul_mat with B2Q_TYPE_F16: fp16 rounding of
the activations, tcgen05 kind::f16 GEMM with fp32 accumulation) against the
oracle's restatement of ggml's CPU path, and the reference's own regression
check for F16 weights (cpp_ggml/src/matmul_backend_test.cpp:24-98,177-183).

Bars: the activation rounding is bit-exact (round to nearest even, as ggml's
fp32 -> fp16 row conversion); the fp32 result within F16_RTOL relative
Frobenius error of the oracle (both sides sum exact fp16 x fp16 products; they
differ only in the fp32 accumulation order of the tensor core)."""
import numpy as np
import pytest

import b2q
import oracle as O
from helpers import reference_check, rel_frobenius, sample

pytestmark = pytest.mark.gpu

F16_RTOL = 1e-5


def to_dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.fixture(autouse=True)
def _no_device_errors(b2q_mod, dev):
    yield
    assert b2q.device_status(clear=True) == 0


@pytest.mark.parametrize("M,N,K", [(1, 1, 8), (31, 65, 256), (33, 65, 256), (129, 130, 72), (300, 257, 1000),
                                   (5, 200, 4096), (700, 384, 1024), (4096, 4096, 1024)])
def test_f16_mul_mat_matches_oracle(dev, M, N, K):
    rng = np.random.default_rng(M * 13 + N * 7 + K)
    w16 = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    y = b2q.mul_mat(b2q.TYPE_F16, to_dev(w16, dev), to_dev(x, dev), bias=to_dev(bias, dev)).cpu().numpy()
    ref = O.mul_mat_f16(w16, x) + bias
    assert np.all(np.isfinite(y))
    assert rel_frobenius(y, ref) <= F16_RTOL


def test_f16_activation_rounding_is_nearest_even(dev):
    """Identity weights return the fp16-rounded activations exactly: ties to
    even, subnormals, the largest finite value."""
    K = 64
    w16 = np.eye(K, dtype=np.float16)
    e = np.float32
    special = [1 + 2 ** -11, 1 + 3 * 2 ** -11, -(1 + 2 ** -11), 2 ** -25, 3 * 2 ** -25, 2 ** -24, 65504.0, 65519.0,
               -65504.0, 0.1, -0.0, 1e-8, 2049.0, 2051.0, 4097.0, 3.14159265]
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((40, K)) * 10).astype(e)
    x[0, :len(special)] = np.array(special, dtype=e)
    y = b2q.mul_mat(b2q.TYPE_F16, to_dev(w16, dev), to_dev(x, dev)).cpu().numpy()
    assert np.array_equal(y, x.astype(np.float16).astype(e))


@pytest.mark.parametrize("M", [31, 32, 33, 65])
def test_f16_reference_regression_check(dev, M):
    """The reference's regression test for F16 weights with F32 input (its GPU
    backends' case): hash inputs, K = 256, N = 65, two iterations on one weight
    buffer, finite outputs, correlation >= 0.9999 and |err| <= 0.05 against
    the fp64 dot of the weights with the fp32 inputs."""
    K, N = 256, 65
    w16 = sample(np.arange(K * N), 13).reshape(N, K).astype(np.float16)
    w_d = to_dev(w16, dev)
    for it in range(2):
        x = sample(np.arange(K * M), 19 + it).reshape(M, K)
        y = b2q.mul_mat(b2q.TYPE_F16, w_d, to_dev(x, dev)).cpu().numpy()
        r = reference_check(y, w16.astype(np.float32), x, it)
        assert r["ok"] and r["max"] <= 0.05, r
        assert rel_frobenius(y, O.mul_mat_f16(w16, x)) <= F16_RTOL


def test_f16_strided_weight_rows_and_output(dev):
    """Row-offset weight views (padded rows) and a strided output view."""
    import torch
    M, N, K = 77, 96, 512
    rng = np.random.default_rng(8)
    wpad = (rng.standard_normal((N + 5, K + 24)) * 0.05).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w_d = to_dev(wpad, dev)[3:3 + N, :K]          # row stride (K + 24) * 2 bytes, 16-byte multiple
    out = torch.full((M, N + 16), float("nan"), device=dev)
    b2q.mul_mat(b2q.TYPE_F16, w_d, to_dev(x, dev), k=K, out=out[:, :N])
    o = out.cpu().numpy()
    assert rel_frobenius(o[:, :N], O.mul_mat_f16(wpad[3:3 + N, :K], x)) <= F16_RTOL
    assert np.all(np.isnan(o[:, N:]))
