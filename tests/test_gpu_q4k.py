"""GPU parity of Q4_K weights (ggml's shipped 4-bit k-quant) against Q8_K
activations, through the C ABI, with the oracle (oracle/b2q_oracle_k.c) as the
checker.  Bars: Q8_K activation codes and scales bit-exact; the three-plane
weight layout equal to its definition from the GGUF bytes; the fp32 mul_mat
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


def test_q4_k_planes_layout(dev):
    """The packed Q4_K weight: planes q*(sc&7), q*(sc>>3), m and fp32 d, dmin,
    computed here from the GGUF bytes with the oracle's unpacking."""
    N, K = 5, 512
    w = O.random_q4_k(N, K, seed=11)
    buf = to_np(b2q.weight_pack(b2q.TYPE_Q4_K, to_dev(w, dev), K))
    planes = buf[:3 * N * K].view(np.int8).reshape(3, N, K)
    ld = (N + 3) // 4 * 4
    o1 = (3 * N * K + 255) // 256 * 256
    o2 = o1 + ((K // 256) * ld * 4 + 255) // 256 * 256
    d = buf[o1:o1 + (K // 256) * ld * 4].view(np.float32).reshape(K // 256, ld)[:, :N]
    dmin = buf[o2:o2 + (K // 256) * ld * 4].view(np.float32).reshape(K // 256, ld)[:, :N]
    blk = w.reshape(N, K // 256, 144)
    for r in range(N):
        for sb in range(K // 256):
            b = blk[r, sb]
            assert d[sb, r] == np.float32(b[0:2].copy().view(np.float16)[0])
            assert dmin[sb, r] == np.float32(b[2:4].copy().view(np.float16)[0])
            for j in range(8):
                if j < 4:     # scales s = b[4:16]: s[j] & 63, s[j+4] & 63
                    sc, m = b[4 + j] & 63, b[8 + j] & 63
                else:         # (s[j+4] & 15) | (s[j-4] >> 6) << 4, (s[j+4] >> 4) | (s[j] >> 6) << 4
                    sc = (b[8 + j] & 15) | ((b[j] >> 6) << 4)
                    m = (b[8 + j] >> 4) | ((b[4 + j] >> 6) << 4)
                grp = b[16 + 32 * (j // 2):16 + 32 * (j // 2) + 32]
                q = (grp & 15) if j % 2 == 0 else (grp >> 4)
                k0 = sb * 256 + 32 * j
                assert np.array_equal(planes[0, r, k0:k0 + 32], (q * (sc & 7)).astype(np.int8))
                assert np.array_equal(planes[1, r, k0:k0 + 32], (q * (sc >> 3)).astype(np.int8))
                assert np.all(planes[2, r, k0:k0 + 32] == m)


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
