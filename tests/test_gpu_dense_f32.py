"""The dequantize-to-float form of the reference's linears (matmul_weight with
keep_quant_gemm false, cpp_ggml/src/ss_flow_graph.cpp:13-34): b2q_dequantize
(ggml_cast of a Q8_0 / Q4_0 / Q4_K weight to F32 or F16) against the oracle's
dequantize_row_* restatement, bit for bit, and b2q_mul_mat_f32 (GGML_PREC_F32
mul_mat on F32 weights, graph_builder.cpp:44-60) against an fp64 product."""
import numpy as np
import pytest

import oracle as O
from helpers import make_case, rel_frobenius

F32_RTOL = 2e-6  # fp32 FMA chain over K <= 4096 vs fp64, relative Frobenius


def _q4k(n, k, seed):
    return O.random_q4_k(n, k, seed)


def _deq_ref(wtype, wq, k):
    return O.dequantize_q4_k(wq, k) if wtype == O.TYPE_Q4_K else O.dequantize(wq, wtype, k)


@pytest.mark.gpu
@pytest.mark.parametrize("wtype", [8, 2, 12])
@pytest.mark.parametrize("out_type", [0, 1])
@pytest.mark.parametrize("n,k", [(1, 256), (37, 512), (300, 1024)])
def test_dequantize_matches_oracle_bitwise(b2q_mod, dev, wtype, out_type, n, k):
    import torch
    wq = _q4k(n, k, 5) if wtype == 12 else make_case(n + k, 1, n, k, wtype)[1]
    ref = _deq_ref(wtype, wq, k)
    got = b2q_mod.dequantize(wtype, torch.from_numpy(np.ascontiguousarray(wq)).to(dev), k, out_type=out_type)
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    if out_type == 1:  # as_f16: the fp32 value rounded once to fp16
        assert np.array_equal(got.view(np.uint16), ref.astype(np.float16).view(np.uint16))
    else:
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert b2q_mod.device_status() == 0


@pytest.mark.gpu
def test_dequantize_row_offset_view_and_padded_output(b2q_mod, dev):
    """A row-range view of the weight (matrix_rows, ss_flow_graph.cpp:38-44)
    into an output with padded rows."""
    import torch
    n, k = 96, 512
    wq = make_case(3, 1, n, k, O.TYPE_Q8_0)[1]
    w_d = torch.from_numpy(wq).to(dev)
    out = torch.full((32, k + 64), -7.0, dtype=torch.float32, device=dev)
    b2q_mod.dequantize(O.TYPE_Q8_0, w_d[40:72], k, out=out[:, :k])
    torch.cuda.synchronize()
    ref = O.dequantize(wq[40:72], O.TYPE_Q8_0, k)
    got = out.cpu().numpy()
    assert np.array_equal(got[:, :k], ref)
    assert np.all(got[:, k:] == -7.0)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(1, 1, 4), (7, 33, 100), (129, 200, 1024), (300, 1000, 640), (64, 128, 4096)])
def test_mul_mat_f32_matches_fp64(b2q_mod, dev, M, N, K):
    import torch
    rng = np.random.default_rng(M * 7 + N + K)
    w = rng.standard_normal((N, K)).astype(np.float32) * 0.05
    x = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    got = b2q_mod.mul_mat_f32(torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev),
                              bias=torch.from_numpy(b).to(dev))
    torch.cuda.synchronize()
    ref = x.astype(np.float64) @ w.astype(np.float64).T + b
    assert rel_frobenius(got.cpu().numpy(), ref) <= F32_RTOL
    assert b2q_mod.device_status() == 0


@pytest.mark.gpu
def test_mul_mat_f32_strided_operands(b2q_mod, dev):
    import torch
    rng = np.random.default_rng(11)
    M, N, K = 100, 70, 256
    wbig = torch.from_numpy(rng.standard_normal((N, K + 32)).astype(np.float32)).to(dev)
    xbig = torch.from_numpy(rng.standard_normal((M, K + 8)).astype(np.float32)).to(dev)
    ybig = torch.full((M, N + 5), 3.0, device=dev)
    b2q_mod.mul_mat_f32(wbig[:, :K], xbig[:, :K], out=ybig[:, :N])
    torch.cuda.synchronize()
    ref = xbig[:, :K].double().cpu().numpy() @ wbig[:, :K].double().cpu().numpy().T
    got = ybig.cpu().numpy()
    assert rel_frobenius(got[:, :N], ref) <= F32_RTOL
    assert np.all(got[:, N:] == 3.0)


@pytest.mark.gpu
@pytest.mark.parametrize("wtype", [8, 2])
def test_as_f32_linear_at_baseline_shape(b2q_mod, dev, wtype):
    """fc1 at BASELINE size through the strict form: dequantize the Q8_0 / Q4_0
    weight to F32, then the F32 mul_mat (+ bias), against fp64 of the oracle's
    dequantized weight."""
    import torch
    M, N, K = 4096, 4096, 1024
    _, wq, x = make_case(17, M, N, K, wtype)
    b = np.random.default_rng(2).standard_normal(N).astype(np.float32)
    wf = b2q_mod.dequantize(wtype, torch.from_numpy(wq).to(dev), K)
    y = b2q_mod.mul_mat_f32(wf, torch.from_numpy(x).to(dev), bias=torch.from_numpy(b).to(dev))
    torch.cuda.synchronize()
    ref = x.astype(np.float64) @ O.dequantize(wq, wtype, K).astype(np.float64).T + b
    assert rel_frobenius(y.cpu().numpy(), ref) <= F32_RTOL


@pytest.mark.gpu
def test_as_f16_linear_matches_oracle(b2q_mod, dev):
    """as_f16: the quantized weight cast to F32 then F16, then the F16 mul_mat."""
    import torch
    M, N, K = 300, 512, 1024
    _, wq, x = make_case(23, M, N, K, O.TYPE_Q4_0)
    w16 = b2q_mod.dequantize(O.TYPE_Q4_0, torch.from_numpy(wq).to(dev), K, out_type=b2q_mod.TYPE_F16)
    y = b2q_mod.mul_mat(b2q_mod.TYPE_F16, w16, torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    ref = O.mul_mat_f16(O.dequantize(wq, O.TYPE_Q4_0, K).astype(np.float16), x)
    assert rel_frobenius(y.cpu().numpy(), ref) <= 1e-5


# ------------------------------------------------------ argument checks (CPU)
FAKE = 1 << 20


@pytest.mark.parametrize("args,expect", [
    ((0, FAKE, 1024, 4, 512, 0, FAKE, 2048), 2),    # F32 "weights" are not a quantized type
    ((8, FAKE, 544, 4, 512, 8, FAKE, 2048), 2),     # output type Q8_0
    ((8, FAKE, 544, 4, 500, 0, FAKE, 2048), 1),     # k % 32
    ((12, FAKE, 288, 4, 288, 0, FAKE, 2048), 1),    # Q4_K k % 256
    ((8, FAKE, 500, 4, 512, 0, FAKE, 2048), 1),     # weight row stride below the row bytes
    ((8, FAKE, 544, 4, 512, 0, FAKE, 2000), 1),     # output row stride below k values
    ((8, FAKE + 1, 544, 4, 512, 0, FAKE, 2048), 3),  # weights not 2-byte aligned
    ((8, FAKE, 544, 4, 512, 0, FAKE + 4, 2048), 3),  # output not 16-byte aligned
])
def test_dequantize_argument_checks(b2q_mod, args, expect):
    assert b2q_mod.lib().b2q_dequantize(*args, None) == expect


@pytest.mark.parametrize("args,expect", [
    ((FAKE, 1024, 4, 254, FAKE, 1024, 8, None, FAKE, 16), 1),   # k % 4
    ((FAKE, 1000, 4, 256, FAKE, 1024, 8, None, FAKE, 16), 1),   # w stride below k floats
    ((FAKE, 1024, 4, 256, FAKE, 1024, 8, None, FAKE, 12), 1),   # y stride below n floats
    ((FAKE + 4, 1024, 4, 256, FAKE, 1024, 8, None, FAKE, 16), 3),  # w not 16-byte aligned
    ((FAKE, 1040, 4, 256, FAKE, 1028, 8, None, FAKE, 16), 3),   # x stride not a multiple of 16 bytes
])
def test_mul_mat_f32_argument_checks(b2q_mod, args, expect):
    assert b2q_mod.lib().b2q_mul_mat_f32(*args, None) == expect
