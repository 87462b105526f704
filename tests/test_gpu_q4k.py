"""GPU parity of Q4_K weights (ggml's shipped 4-bit k-quant) against Q8_K
activations, through the C ABI, with the oracle (oracle/b2q_oracle_k.c) as the
checker.  Bars: Q8_K activation codes and scales bit-exact; the three-plane
packed weight equal to the GGUF rows; the fp32 mul_mat
within RTOL (relative Frobenius) of the oracle's ggml-order dot."""
import numpy as np
import pytest

import b2q
import oracle as O
from helpers import rel_frobenius

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def to_dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def to_np(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(autouse=True)
def _no_device_errors(b2q_mod, dev):
    yield
    assert b2q.device_status(clear=True) == 0


@pytest.mark.parametrize("M,K", [(1, 256), (37, 1024), (300, 4096)])
def test_q8_k_activations_bit_exact(dev, M, K):
    """Prepared Q8_K activations (codes [M][K], fp32 d [K/256][ld]) equal the
    oracle's block_q8_K codes and d."""
    rng = np.random.default_rng(M + K)
    x = (rng.standard_normal((M, K)) * rng.uniform(0.01, 10, (M, 1))).astype(np.float32)
    x[0, :256] = 0.0                       # all-zero block
    if M > 1:
        x[1, 3], x[1, 7] = 5.0, -5.0       # |x| tie: the first one sets the sign
    act = to_np(b2q.act_prepare(to_dev(x, dev), b2q.ACT_Q8_K))
    assert act.size == b2q.act_prepared_bytes(b2q.ACT_Q8_K, M, K)
    codes = act[:M * K].view(np.int8).reshape(M, K)
    off, ld = (M * K + 255) // 256 * 256, (M + 3) // 4 * 4
    d = act[off:off + (K // 256) * ld * 4].view(np.float32).reshape(K // 256, ld)[:, :M]
    ref = O.quantize_q8_k(x).reshape(M, K // 256, 292)
    assert np.array_equal(codes.reshape(M, K // 256, 256), ref[:, :, 4:260].view(np.int8))
    assert np.array_equal(d.T.view(np.uint32), ref[:, :, :4].copy().view(np.uint32)[:, :, 0])


def test_q4_k_packed_is_the_gguf_rows(dev):
    """The packed Q4_K weight is the block_q4_K rows themselves, contiguous
    (the kernel unpacks them on chip), from a strided row view too."""
    import torch
    N, K = 5, 512
    w = O.random_q4_k(N, K, seed=11)
    wide = np.zeros((N, w.shape[1] + 32), np.uint8)
    wide[:, 16:16 + w.shape[1]] = w
    buf = to_np(b2q.weight_pack(b2q.TYPE_Q4_K, to_dev(wide, dev)[:, 16:16 + w.shape[1]], K))
    assert buf.size == b2q.weight_packed_bytes(b2q.TYPE_Q4_K, N, K)
    assert np.array_equal(buf[:w.size].reshape(N, -1), w)
    torch.cuda.synchronize()


@pytest.mark.parametrize("M,N,K", [(300, 200, 1024), (4, 1000, 2048), (1, 64, 256), (129, 3072, 1024)])
def test_q4_k_mul_mat_matches_oracle(dev, M, N, K):
    w = O.random_q4_k(N, K, seed=N + K)
    x = np.random.default_rng(M * 3 + K).standard_normal((M, K)).astype(np.float32)
    y = to_np(b2q.mul_mat(b2q.TYPE_Q4_K, to_dev(w, dev), to_dev(x, dev)))
    assert rel_frobenius(y, O.mul_mat_q4_k(w, x)) <= RTOL


def test_q4_k_packed_and_prepared_paths_agree(dev):
    """Raw, packed (variant Q8_K), prepared, uploaded and gated-residual entry
    points agree bit for bit, including a few-token call."""
    import torch
    M, N, K = 70, 512, 1024
    w = O.random_q4_k(N, K, seed=3)
    x = np.random.default_rng(4).standard_normal((M, K)).astype(np.float32)
    w_d, x_d = to_dev(w, dev), to_dev(x, dev)
    bias = torch.randn(N, device=dev)
    y_raw = b2q.mul_mat(b2q.TYPE_Q4_K, w_d, x_d, bias=bias)
    packed = b2q.weight_pack(b2q.TYPE_Q4_K, w_d, K)
    y_pk = b2q.mul_mat_packed(packed, N, K, x_d, bias=bias, variant=b2q.ACT_Q8_K)
    act = b2q.act_prepare(x_d, b2q.ACT_Q8_K)
    y_pr = b2q.mul_mat_prepared_q4_k(packed, N, K, act, M, bias=bias)
    up = b2q.weight_upload(b2q.TYPE_Q4_K, w, K, staging_bytes=144 * 4 * 9, device=dev)
    y_up = b2q.mul_mat_prepared_q4_k(up, N, K, act, M, bias=bias)
    r = torch.randn(M, N, device=dev)
    g = torch.randn(N, device=dev)
    z = b2q.mul_mat_prepared_q4_k(packed, N, K, act, M, bias=bias, gate=g, resid=r)
    r2 = r.clone()
    b2q.mul_mat_prepared_q4_k(packed, N, K, act, M, bias=bias, gate=g, resid=r2, out=r2)
    act4 = b2q.act_prepare(x_d[:4].contiguous(), b2q.ACT_Q8_K)
    y4 = b2q.mul_mat_prepared_q4_k(packed, N, K, act4, 4, bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(y_raw, y_pk) and torch.equal(y_raw, y_pr) and torch.equal(y_raw, y_up)
    assert torch.equal(z, r + y_raw * g) and torch.equal(r2, z)
    assert torch.equal(y4, y_raw[:4])
    assert rel_frobenius(to_np(y_raw) - to_np(bias)[None, :], O.mul_mat_q4_k(w, x)) <= RTOL
