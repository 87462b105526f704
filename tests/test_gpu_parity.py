"""GPU parity of the CUDA path against the CPU oracle, through the C ABI.

Bars: quantize bytes bit-exact; int32 per-block dots
bit-exact; fp32 mul_mat within relative Frobenius error 1e-5 of the ggml CPU
semantics (RTOL below).  The CUDA-core check kernel must also be bit-exact in
fp32 because it follows the CPU's accumulation order."""
import numpy as np
import pytest

import b2q
import oracle as O
from helpers import gelu_tanh, make_case, reference_check, rel_frobenius, sample

pytestmark = pytest.mark.gpu

RTOL = 1e-5  # relative Frobenius tolerance of the fp32 result


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


# ------------------------------------------------------------------ quantize
@pytest.mark.parametrize("variant", [O.ACT_X86, O.ACT_REF])
@pytest.mark.parametrize("M,K", [(1, 32), (33, 256), (7, 96), (1374, 1024), (4096, 1024)])
def test_quantize_bit_exact(dev, variant, M, K):
    rng = np.random.default_rng(M * 7 + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[0, :32] = 0.0
    if M > 3:
        x[1, :32] = np.arange(32, dtype=np.float32) - 15.5
        x[2, :32] = 1e-30
        x[3, :32] = 3e4 * rng.standard_normal(32)
    got = to_np(b2q.quantize_q8_0(to_dev(x, dev), variant))
    assert np.array_equal(got, O.quantize(x, O.TYPE_Q8_0, variant))


def test_quantize_unaligned_rows_use_scalar_loads(dev):
    import torch
    rng = np.random.default_rng(5)
    big = rng.standard_normal((9, 1024 + 3)).astype(np.float32)
    xb = to_dev(big, dev)
    x = xb[:, 1:1 + 1024]                       # 4-byte aligned, not 16
    got = to_np(b2q.quantize_q8_0(x, O.ACT_X86))
    assert np.array_equal(got, O.quantize(big[:, 1:1 + 1024], O.TYPE_Q8_0, O.ACT_X86))
    del torch


def test_quantize_golden_ref_variant(dev):
    g = np.load(__file__.replace("test_gpu_parity.py", "golden/q_golden.npz"))
    got = to_np(b2q.quantize_q8_0(to_dev(g["x"], dev), O.ACT_REF))
    assert np.array_equal(got, g["a_q8_ref"])


# ---------------------------------------------------------------- block dots
@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M,N,K", [(1, 1, 32), (33, 65, 256), (129, 257, 96), (200, 130, 4096),
                                   (300, 128, 160)])
def test_tensor_core_block_dots_bit_exact(dev, wtype, M, N, K):
    _, wq, x = make_case(M + N + K, M, N, K, wtype)
    a = O.quantize(x, O.TYPE_Q8_0, O.ACT_X86)
    got = to_np(b2q.block_dots(wtype, to_dev(wq, dev), to_dev(a, dev), K))
    assert np.array_equal(got, O.block_dots(wtype, wq, a, K))


@pytest.mark.parametrize("name,wtype", [("q8_0", O.TYPE_Q8_0), ("q4_0", O.TYPE_Q4_0)])
def test_block_dots_golden(dev, name, wtype):
    g = np.load(__file__.replace("test_gpu_parity.py", "golden/q_golden.npz"))
    K = int(g["K"])
    got = to_np(b2q.block_dots(wtype, to_dev(g[f"w_{name}"], dev), to_dev(g["a_q8_ref"], dev), K))
    assert np.array_equal(got, g[f"dots_{name}"])


# ------------------------------------------------------- CUDA-core check path
@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M,N,K", [(1, 1, 32), (33, 65, 256), (65, 100, 1024), (17, 40, 4096)])
def test_simt_fp32_bit_exact(dev, wtype, M, N, K):
    _, wq, x = make_case(3 * M + N + K, M, N, K, wtype)
    a = O.quantize(x, O.TYPE_Q8_0, O.ACT_X86)
    got = to_np(b2q.mul_mat_q_simt(wtype, to_dev(wq, dev), to_dev(a, dev), K))
    ref = O.mul_mat_q(wtype, wq, a, K)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


# ----------------------------------------------------------- tcgen05 mul_mat
SHAPES = [(1, 64, 32), (31, 65, 256), (32, 65, 256), (33, 65, 256), (65, 65, 256),
          (127, 129, 96), (128, 128, 128), (129, 257, 1024), (256, 384, 224),
          (1374, 1024, 1024)]


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_mul_mat_matches_oracle(dev, wtype, M, N, K):
    _, wq, x = make_case(M * 31 + N * 7 + K, M, N, K, wtype)
    y = to_np(b2q.mul_mat(wtype, to_dev(wq, dev), to_dev(x, dev)))
    ref = O.mul_mat(wtype, wq, x, O.ACT_X86)
    assert np.all(np.isfinite(y))
    assert rel_frobenius(y, ref) <= RTOL


# The GEMM picks its tile width (tokens per tile) per shape; on a 148-SM B200
# these shapes select 80, 96, 112 and 128 respectively, each with a ragged
# last token tile.  Bias and a padded output row pitch ride along.
@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M,N,K", [(912, 1280, 256), (1136, 1280, 256), (1360, 1280, 256), (1584, 1280, 256)])
def test_every_tile_width_matches_oracle(dev, wtype, M, N, K):
    import torch
    _, wq, x = make_case(M + N + K, M, N, K, wtype)
    bias = np.random.default_rng(M).standard_normal(N).astype(np.float32)
    out = torch.full((M, N + 8), float("nan"), dtype=torch.float32, device=dev)
    b2q.mul_mat(wtype, to_dev(wq, dev), to_dev(x, dev), bias=to_dev(bias, dev), out=out[:, :N])
    got = to_np(out)
    ref = O.mul_mat(wtype, wq, x, O.ACT_X86) + bias[None, :]
    assert np.all(np.isnan(got[:, N:]))  # nothing written past the row
    assert rel_frobenius(got[:, :N], ref) <= RTOL


@pytest.mark.parametrize("wtype,M,N,K,gelu", [
    (O.TYPE_Q8_0, 4096, 4096, 1024, False),    # fc1, Q8_0
    (O.TYPE_Q4_0, 4096, 4096, 1024, False),    # fc1, Q4_0
    (O.TYPE_Q4_0, 4096, 1024, 4096, True),     # fc2, Q4_0, GELU inputs
    (O.TYPE_Q8_0, 1374, 1024, 1024, False),    # small-M cross-attention kv
])
def test_baseline_shapes_match_oracle(dev, wtype, M, N, K, gelu):
    _, wq, x = make_case(M + N + K + gelu, M, N, K, wtype, gelu=gelu)
    y = to_np(b2q.mul_mat(wtype, to_dev(wq, dev), to_dev(x, dev)))
    ref = O.mul_mat(wtype, wq, x, O.ACT_X86)
    assert rel_frobenius(y, ref) <= RTOL


@pytest.mark.parametrize("variant", [O.ACT_X86, O.ACT_REF])
def test_variants_follow_oracle(dev, variant):
    _, wq, x = make_case(99, 200, 96, 512, O.TYPE_Q8_0)
    y = to_np(b2q.mul_mat(O.TYPE_Q8_0, to_dev(wq, dev), to_dev(x, dev), variant=variant))
    assert rel_frobenius(y, O.mul_mat(O.TYPE_Q8_0, wq, x, variant)) <= RTOL


def test_packed_path_bitwise_equals_raw_path(dev):
    import torch
    M, N, K = 300, 200, 640
    _, wq, x = make_case(7, M, N, K, O.TYPE_Q4_0)
    w_d, x_d = to_dev(wq, dev), to_dev(x, dev)
    packed = b2q.weight_pack(O.TYPE_Q4_0, w_d, K)
    y1 = b2q.mul_mat_packed(packed, N, K, x_d)
    y0 = b2q.mul_mat(O.TYPE_Q4_0, w_d, x_d)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


def test_bias_is_fused_add(dev):
    import torch
    M, N, K = 129, 300, 256
    _, wq, x = make_case(8, M, N, K, O.TYPE_Q8_0)
    bias = np.random.default_rng(1).standard_normal(N).astype(np.float32)
    w_d, x_d = to_dev(wq, dev), to_dev(x, dev)
    y0 = b2q.mul_mat(O.TYPE_Q8_0, w_d, x_d)
    y1 = b2q.mul_mat(O.TYPE_Q8_0, w_d, x_d, bias=to_dev(bias, dev))
    torch.cuda.synchronize()
    # mul_mat then GGML_OP_ADD in fp32 == fused epilogue add, bit for bit
    assert torch.equal(y1, y0 + to_dev(bias, dev))


def test_row_offset_view_and_strided_output(dev):
    """matrix_rows (cpp_ggml/src/ss_flow_graph.cpp:38-44): src0 is a row range of
    a fused qkv weight; dst rows are written with a stride wider than N."""
    import torch
    C, K, M = 96, 256, 70
    _, wq, x = make_case(12, M, 3 * C, K, O.TYPE_Q8_0)
    w_d, x_d = to_dev(wq, dev), to_dev(x, dev)
    out = torch.full((M, 2 * C + 8), -7.0, dtype=torch.float32, device=dev)
    kview = w_d[C:2 * C]                       # rows C..2C-1, row stride = full row bytes
    b2q.mul_mat(O.TYPE_Q8_0, kview, x_d, out=out[:, 4:4 + C])
    y = to_np(out)
    ref = O.mul_mat(O.TYPE_Q8_0, wq[C:2 * C], x, O.ACT_X86)
    assert rel_frobenius(y[:, 4:4 + C], ref) <= RTOL
    assert np.all(y[:, :4] == -7.0) and np.all(y[:, 4 + C:] == -7.0)


def test_repeat_calls_are_deterministic(dev):
    import torch
    _, wq, x = make_case(13, 1000, 512, 1024, O.TYPE_Q8_0)
    w_d, x_d = to_dev(wq, dev), to_dev(x, dev)
    y0 = b2q.mul_mat(O.TYPE_Q8_0, w_d, x_d)
    y1 = b2q.mul_mat(O.TYPE_Q8_0, w_d, x_d)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M", [31, 32, 33, 65])
def test_reference_regression_check(dev, wtype, M):
    """The reference's matmul regression test, run through the C ABI: hash
    inputs, K = 256, N = 65, two iterations on the same weight buffer
    (cpp_ggml/src/matmul_backend_test.cpp:24-98; criteria in helpers)."""
    K, N = 256, 65
    w = sample(np.arange(K * N), 13).reshape(N, K)
    wq = O.quantize(w, wtype)
    w_deq = O.dequantize(wq, wtype, K)
    w_d = to_dev(wq, dev)
    for it in range(2):
        x = sample(np.arange(K * M), 19 + it).reshape(M, K)
        y = to_np(b2q.mul_mat(wtype, w_d, to_dev(x, dev)))
        r = reference_check(y, w_deq, x, it)
        assert r["ok"], r
        assert rel_frobenius(y, O.mul_mat(wtype, wq, x, O.ACT_X86)) <= RTOL


def test_gelu_inputs_large_k(dev):
    # fc2-like: GELU(N(0,1)) activations, K = 4096, ragged N
    _, wq, x = make_case(21, 300, 200, 4096, O.TYPE_Q8_0, gelu=True)
    y = to_np(b2q.mul_mat(O.TYPE_Q8_0, to_dev(wq, dev), to_dev(x, dev)))
    assert rel_frobenius(y, O.mul_mat(O.TYPE_Q8_0, wq, x, O.ACT_X86)) <= RTOL
    assert np.allclose(gelu_tanh(np.zeros(1, np.float32)), 0)


# ---------------------------------------------------- few tokens (M <= 8)
@pytest.mark.parametrize("wtype,N,K", [
    (O.TYPE_Q8_0, 6144, 1024),   # adaLN projection, M = 1 per sample (ss_flow_graph.cpp:183-185)
    (O.TYPE_Q4_0, 1024, 4096),   # pose-group fc2, M = 4
    (O.TYPE_Q4_0, 1003, 96),     # ragged rows, 3 blocks
    (O.TYPE_Q8_0, 72, 8192),     # two K chunks
])
def test_few_tokens_bit_identical_to_tensor_core_path(dev, wtype, N, K):
    """M <= 8 runs on the CUDA-core kernel; its rows equal the tensor-core
    kernel's rows for the same tokens bit for bit (bias, gate and residual
    included), and the oracle within RTOL."""
    import torch
    big = 64
    _, wq, xb = make_case(N + K, big, N, K, wtype)
    rng = np.random.default_rng(K)
    bias = rng.standard_normal(N).astype(np.float32)
    gate = rng.standard_normal(N).astype(np.float32)
    resid = rng.standard_normal((big, N)).astype(np.float32)
    packed = b2q.weight_pack(wtype, to_dev(wq, dev), K)
    b_d, g_d, r_d = to_dev(bias, dev), to_dev(gate, dev), to_dev(resid, dev)
    xb_d = to_dev(xb, dev)
    act_b = b2q.act_prepare(xb_d)
    y_tc = b2q.mul_mat_prepared(packed, N, K, act_b, big, bias=b_d)
    z_tc = b2q.mul_mat_prepared_gate_residual(packed, N, K, act_b, big, r_d, bias=b_d, gate=g_d)
    for M in (1, 2, 3, 4, 5, 8):
        act = b2q.act_prepare(xb_d[:M].contiguous())
        y = b2q.mul_mat_prepared(packed, N, K, act, M, bias=b_d)
        z = b2q.mul_mat_prepared_gate_residual(packed, N, K, act, M, r_d[:M].contiguous(), bias=b_d, gate=g_d)
        torch.cuda.synchronize()
        assert torch.equal(y, y_tc[:M]), M
        assert torch.equal(z, z_tc[:M]), M
    y1 = to_np(b2q.mul_mat(wtype, to_dev(wq, dev), xb_d[:3].contiguous()))
    assert rel_frobenius(y1, O.mul_mat(wtype, wq, xb[:3], O.ACT_X86)) <= RTOL


@pytest.mark.parametrize("wtype,N,K,staging", [
    (O.TYPE_Q8_0, 1000, 1024, 34 * 32 * 7),      # 7 rows per chunk, ragged last chunk
    (O.TYPE_Q4_0, 4096, 1024, 8 << 20),          # one chunk
    (O.TYPE_Q4_0, 65, 256, 18 * 8),              # one row per chunk
])
def test_weight_upload_from_host_equals_device_pack(dev, wtype, N, K, staging):
    """Host GGUF rows (strided: a row-offset view of a wider tensor) uploaded in
    chunks through a small staging buffer pack to the same bytes as packing the
    rows already on the device, and serve mul_mat identically."""
    import torch
    _, wq, x = make_case(N + 3 * K, 40, N, K, wtype)
    rb = wq.shape[1]
    host = np.zeros((N, rb + 6), np.uint8)
    host[:, 2:2 + rb] = wq
    view = host[:, 2:2 + rb]
    p_up = b2q.weight_upload(wtype, view, K, staging_bytes=staging, device=dev)
    p_dev = b2q.weight_pack(wtype, to_dev(wq, dev), K)
    torch.cuda.synchronize()
    off, ld = (N * K + 255) // 256 * 256, (N + 3) // 4 * 4   # codes [N][K], then scales [K/32][ld]
    a, b = to_np(p_up), to_np(p_dev)
    assert np.array_equal(a[:N * K], b[:N * K])
    sa = a[off:off + (K // 32) * ld * 4].view(np.float32).reshape(K // 32, ld)[:, :N]
    sb = b[off:off + (K // 32) * ld * 4].view(np.float32).reshape(K // 32, ld)[:, :N]
    assert np.array_equal(sa.view(np.uint32), sb.view(np.uint32))
    x_d = to_dev(x, dev)
    assert torch.equal(b2q.mul_mat_packed(p_up, N, K, x_d), b2q.mul_mat_packed(p_dev, N, K, x_d))
