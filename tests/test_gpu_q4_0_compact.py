"""Compact Q4_0 weights (the GGUF footprint, nibbles widened on chip) against
the int8 layout of the same weight and against the oracle: the GEMM sees the
same int8 codes and fp32 scales either way, so the outputs are equal bit for
bit; the compact buffer is 0.5625 bytes per value plus padding."""
import numpy as np
import pytest

import b2q
import colpar
import oracle as O
from helpers import make_case, rel_frobenius


def test_compact_q4_0_size_is_the_gguf_footprint(b2q_mod):
    n, k = 4096, 1024
    size = b2q.lib().b2q_weight_packed_q4_0_bytes(n, k)
    assert size == n * k // 2 + (k // 32) * n * 2  # 256-byte padding adds nothing at this shape
    assert size / (n * k) == 0.5625
    assert b2q.lib().b2q_weight_packed_q4_0_bytes(n, 100) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(4096, 4096, 1024), (4096, 1024, 4096), (1374, 1024, 1024), (300, 200, 640),
                                   (5, 72, 96), (129, 131, 2080)])
def test_compact_q4_0_equals_the_int8_layout(b2q_mod, dev, M, N, K):
    import torch
    _, wq, x = make_case(M + N + K, M, N, K, O.TYPE_Q4_0)
    w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
    x_d = torch.from_numpy(x).to(dev)
    rng = np.random.default_rng(N)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
    act = b2q.act_prepare(x_d)
    wide = b2q.weight_pack(O.TYPE_Q4_0, w_d, K)
    comp = b2q.weight_pack_q4_0(w_d, K)
    y_ref = b2q.mul_mat_prepared(wide, N, K, act, M, bias=bias)
    y = b2q.mul_mat_prepared_q4_0(comp, N, K, act, M, bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    if M * N * K <= (1 << 27):
        assert rel_frobenius(y.cpu().numpy() - bias.cpu().numpy(), O.mul_mat(O.TYPE_Q4_0, wq, x, O.ACT_X86)) <= 1e-5
    assert b2q.device_status() == 0


@pytest.mark.gpu
def test_compact_q4_0_fused_tile_ends(b2q_mod, dev):
    import torch
    M, N, K = 513, 1024, 512
    _, wq, x = make_case(7, M, N, K, O.TYPE_Q4_0)
    w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
    act = b2q.act_prepare(torch.from_numpy(x).to(dev))
    wide, comp = b2q.weight_pack(O.TYPE_Q4_0, w_d, K), b2q.weight_pack_q4_0(w_d, K)
    g = torch.Generator(device=dev).manual_seed(1)
    bias, gate = torch.randn(N, device=dev, generator=g), torch.randn(N, device=dev, generator=g)
    r = torch.randn(M, N, device=dev, generator=g)
    z_ref = b2q.mul_mat_prepared_gate_residual(wide, N, K, act, M, r, bias=bias, gate=gate)
    z = b2q.mul_mat_prepared_q4_0(comp, N, K, act, M, bias=bias, gate=gate, resid=r)
    q_ref = b2q.mul_mat_prepared_gelu_q8(wide, N, K, act, M, bias=bias)
    q = b2q.mul_mat_prepared_q4_0_gelu_q8(comp, N, K, act, M, bias=bias)
    r2 = r.clone()
    b2q.mul_mat_prepared_q4_0(comp, N, K, act, M, bias=bias, gate=gate, resid=r2, out=r2)
    torch.cuda.synchronize()
    assert torch.equal(z, z_ref) and torch.equal(r2, z_ref)
    # the prepared activations' written bytes: codes [M][N], scales [N/32][:M]
    # (the layout's 256-byte and 4-row padding is never written)
    qc, qs = colpar.split_views(q, M, N)
    rc, rs = colpar.split_views(q_ref, M, N)
    assert torch.equal(qc, rc) and torch.equal(qs[:, :M], rs[:, :M])
    assert b2q.device_status() == 0
