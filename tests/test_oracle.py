"""CPU tests of the oracle: pinned against gguf-py's golden vectors and the
reference test's pass criteria.  No GPU."""
import os

import numpy as np
import pytest

import oracle as O
from helpers import make_case, reference_check, rel_frobenius, sample

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q_golden.npz")


@pytest.fixture(scope="module")
def golden(oracle_mod):
    return np.load(GOLDEN)


def test_fp16_rounding_matches_ieee(oracle_mod):
    rng = np.random.default_rng(0)
    parts = [rng.standard_normal(20000).astype(np.float32) * s
             for s in (1e-9, 3e-8, 1e-6, 6e-5, 1e-3, 1.0, 300.0, 6e4, 7e4)]
    edge = np.array([0.0, -0.0, 65504, 65519.996, 65520, -65520, 6.1035156e-05, 5.9604645e-08,
                     2.9802322e-08, 2.9802326e-08, 8.940697e-08, np.inf, -np.inf], np.float32)
    x = np.concatenate(parts + [edge])
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(O.fp32_to_fp16_bits(x), ref)


def test_philox_known_answer(oracle_mod):
    # Random123 known-answer vector for philox4x32_10, key 0, counter 0.
    assert [int(v) for v in O.philox(0, 0)] == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_normal_generator_moments(oracle_mod):
    z = O.normal(1 << 18, seed=7)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert np.array_equal(z, O.normal(1 << 18, seed=7))


@pytest.mark.parametrize("name,wtype", [("q8_0", O.TYPE_Q8_0), ("q4_0", O.TYPE_Q4_0)])
def test_weight_quantizer_matches_golden(golden, name, wtype):
    mine = O.quantize(golden["w"], wtype)
    assert np.array_equal(mine, golden[f"w_{name}"])
    K = int(golden["K"])
    assert np.array_equal(O.dequantize(mine, wtype, K), golden[f"w_{name}_dequant"])


REF_Q4 = os.path.join(os.path.dirname(__file__), "golden", "ref_q4_0.npz")


def test_q4_0_quantizer_matches_reference_fixture(oracle_mod):
    """Q4_0 bytes equal the reference's own quantizer (cpp_ggml/scripts/
    gguf_schema.py:27-52, documented there as ggml's quantize_row_q4_0_ref
    byte for byte), recorded by tests/golden/make_ref_q4_golden.py: edge blocks
    in full, and the BASELINE fc1 / fc2 weight shapes by SHA-256."""
    import hashlib
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    try:
        import make_ref_q4_golden as G
    finally:
        sys.path.pop(0)
    g = np.load(REF_Q4)
    assert np.array_equal(O.quantize(g["w_small"], O.TYPE_Q4_0), g["q4_small"])
    for name, n, k, seed in G.BIG:
        assert [int(v) for v in g[f"{name}_shape"]] == [n, k, seed]
        wb = O.quantize(G.big_matrix(n, k, seed), O.TYPE_Q4_0)
        assert np.array_equal(wb[:16], g[f"{name}_head"])
        assert hashlib.sha256(wb.tobytes()).hexdigest() == str(g[f"{name}_sha256"])


def test_q4_0_quantizer_matches_reference_live(oracle_mod):
    """The same pin run live against the reference checkout when it is present
    (this container; the GPU box has none), on fresh seeds and odd scales."""
    import sys
    root = os.path.join(os.sep, "root", "reference", "cpp_ggml", "scripts")
    if not os.path.exists(os.path.join(root, "gguf_schema.py")):
        pytest.skip("reference checkout not present")
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    try:
        import make_ref_q4_golden as G
    finally:
        sys.path.pop(0)
    ref_q4 = G.load_reference_quantizer(os.path.join(os.sep, "root", "reference"))
    rng = np.random.default_rng(99)
    for scale in (1e-5, 0.02, 1.0, 1e4):
        w = (rng.standard_normal((48, 512)) * scale).astype(np.float32)
        w[0, :32] = np.round(w[0, :32] * 8) / 8  # many exact ties
        assert np.array_equal(O.quantize(w, O.TYPE_Q4_0), ref_q4(w).reshape(48, -1))


def test_bench_weights_use_the_ggml_reference_quantizers(oracle_mod):
    """bench.py builds its synthetic GGUF weights in numpy; they must be the
    bytes of the ggml reference quantizers the oracle restates (and, for Q4_0,
    the reference's own quantizer pins)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "bench_mod", os.path.join(os.path.dirname(os.path.dirname(__file__)), "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    rng = np.random.default_rng(5)
    for scale in (0.02, 1.0):
        w = (rng.standard_normal((64, 1024)) * scale).astype(np.float32)
        w[0, :32] = 0.0
        w[1, :32] = np.arange(32, dtype=np.float32) - 15.5
        w[2, 32:64] = np.round(w[2, 32:64] * 127) / 127
        for wtype in (O.TYPE_Q8_0, O.TYPE_Q4_0):
            assert np.array_equal(bench.synth_blocks(wtype, w, 64, 1024), O.quantize(w, wtype))


def test_activation_ref_variant_matches_golden(golden):
    assert np.array_equal(O.quantize(golden["x"], O.TYPE_Q8_0, O.ACT_REF), golden["a_q8_ref"])


def test_activation_variants_share_scales_and_nearly_all_codes(golden):
    x = golden["x"]
    a_x86 = O.quantize(x, O.TYPE_Q8_0, O.ACT_X86).reshape(x.shape[0], -1, 34)
    a_ref = O.quantize(x, O.TYPE_Q8_0, O.ACT_REF).reshape(x.shape[0], -1, 34)
    assert np.array_equal(a_x86[:, :, :2], a_ref[:, :, :2])       # d = amax/127 in both
    diff = a_x86[:, :, 2:].view(np.int8).astype(int) - a_ref[:, :, 2:].view(np.int8).astype(int)
    assert np.all(np.abs(diff) <= 1)                              # only rounding ties differ
    # the planted exact-tie block (x = j - 15.5, amax 15.5 -> |x|*127/15.5 has no .5 ties
    # in fp32, but 1/d vs 127/amax rounding can still move a code by one)
    assert np.mean(diff != 0) < 0.01


@pytest.mark.parametrize("name,wtype", [("q8_0", O.TYPE_Q8_0), ("q4_0", O.TYPE_Q4_0)])
def test_block_dots_match_golden(golden, name, wtype):
    K = int(golden["K"])
    dots = O.block_dots(wtype, golden[f"w_{name}"], golden["a_q8_ref"], K)
    assert np.array_equal(dots, golden[f"dots_{name}"])


@pytest.mark.parametrize("name,wtype", [("q8_0", O.TYPE_Q8_0), ("q4_0", O.TYPE_Q4_0)])
def test_mul_mat_matches_golden_products(golden, name, wtype):
    K = int(golden["K"])
    y = O.mul_mat_q(wtype, golden[f"w_{name}"], golden["a_q8_ref"], K)
    # fp32 accumulation of the exact per-block products: within 1e-6 of fp64
    assert rel_frobenius(y, golden[f"y_blockscale_{name}"]) < 1e-6
    assert rel_frobenius(y, golden[f"y_f64_{name}"]) < 1e-6


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M,N,K", [(1, 1, 32), (31, 65, 256), (33, 17, 96), (65, 130, 1024)])
def test_fast_variant_bit_identical(wtype, M, N, K):
    _, wq, x = make_case(M * 1000 + N + K, M, N, K, wtype)
    a = O.quantize(x, O.TYPE_Q8_0, O.ACT_X86)
    y0 = O.mul_mat_q(wtype, wq, a, K, fast=False)
    y1 = O.mul_mat_q(wtype, wq, a, K, fast=True, nthreads=3)
    assert np.array_equal(y0.view(np.uint32), y1.view(np.uint32))
    yq = O.mul_mat(wtype, wq, x, O.ACT_X86, fast=True)
    assert np.array_equal(y0.view(np.uint32), yq.view(np.uint32))


def test_single_vec_dot_lane_order():
    # one block where lane order matters: d*partial products accumulate per lane
    rng = np.random.default_rng(3)
    _, wq, x = make_case(11, 1, 1, 4096, O.TYPE_Q8_0)
    a = O.quantize(x, O.TYPE_Q8_0, O.ACT_X86)
    y = O.mul_mat_q(O.TYPE_Q8_0, wq, a, 4096)
    f64 = O.mul_mat_f64(O.TYPE_Q8_0, wq, a, 4096)
    assert abs(float(y[0, 0]) - f64[0, 0]) <= 1e-5 * max(1.0, abs(f64[0, 0]))
    del rng


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
@pytest.mark.parametrize("M", [31, 32, 33, 65])
def test_reference_test_criteria_on_oracle(wtype, M):
    """The reference's regression check (matmul_backend_test.cpp:24-98), shapes
    M in {31,32,33,65}, K = 256, N = 65, two iterations, applied to the oracle's
    quantized mul_mat (ggml's CPU path for Q8_0 / Q4_0 weights)."""
    K, N = 256, 65
    w = sample(np.arange(K * N), 13).reshape(N, K)
    wq = O.quantize(w, wtype)
    w_deq = O.dequantize(wq, wtype, K)
    for it in range(2):
        x = sample(np.arange(K * M), 19 + it).reshape(M, K)
        y = O.mul_mat(wtype, wq, x, O.ACT_X86)
        r = reference_check(y, w_deq, x, it)
        assert r["ok"], r


def test_zero_and_degenerate_rows():
    K = 64
    x = np.zeros((3, K), np.float32)
    x[1, :32] = 1e-30          # underflows to a zero fp16 scale
    x[2, :] = -0.0
    a = O.quantize(x, O.TYPE_Q8_0, O.ACT_X86).reshape(3, -1, 34)
    assert np.all(a[:, :, :2] == 0)          # every fp16 scale is zero
    assert np.all(a[0, :, 2:] == 0) and np.all(a[2, :, 2:] == 0)
    # 1e-30: d = amax/127 underflows in fp16 but the fp32 inverse does not,
    # so ggml stores codes of 127 next to a zero scale.
    assert np.all(a[1, 0, 2:].view(np.int8) == 127)
    w = np.ones((2, K), np.float32)
    y = O.mul_mat(O.TYPE_Q8_0, O.quantize(w, O.TYPE_Q8_0), x, O.ACT_X86)
    assert np.all(y == 0)


def test_gelu_table_follows_the_tanh_formula():
    """ggml's fp16 GELU table (restated in the oracle) against the same tanh
    form in fp64: each entry within one fp16 step of the fp64 value plus the
    fp32 formula's own error (1 + tanh cancels for x < 0: a few fp32 ulps of 1,
    times 0.5|x|), 0 / identity outside (-10, 10), NaN through, and the
    contracted (FMA) build of the table differs from the uncontracted one in
    few entries."""
    h = np.arange(65536, dtype=np.uint16)
    fin = np.isfinite(h.view(np.float16)) & (np.abs(h.view(np.float16)) < 10)
    f = h[fin].view(np.float16).astype(np.float64)
    t = O.gelu_table(False)[fin].view(np.float16).astype(np.float64)
    exact = 0.5 * f * (1.0 + np.tanh(0.7978845608028654 * f * (1.0 + 0.044715 * f * f)))
    step = np.abs(np.spacing(exact.astype(np.float16)).astype(np.float64))
    assert np.all(np.abs(t - exact) <= step + 0.5 * np.abs(f) * 4 * 2.0 ** -24)
    assert np.count_nonzero(O.gelu_table(False) != O.gelu_table(True)) <= 8
    x = np.array([-np.inf, -1e6, -10.0, -9.99, 9.99, 10.0, 1e6, np.inf, np.nan, 0.0], np.float32)
    y = O.gelu(x)
    assert list(y[:3]) == [0.0, 0.0, 0.0] and list(y[5:8]) == [10.0, 1e6, np.inf]
    assert np.isnan(y[8]) and y[9] == 0.0
    # inside (-10, 10): x rounded to fp16, then the table entry
    xs = np.random.default_rng(3).uniform(-9.9, 9.9, 4096).astype(np.float32)
    idx = xs.astype(np.float16).view(np.uint16)
    assert np.array_equal(O.gelu(xs), O.gelu_table(False)[idx].view(np.float16).astype(np.float32))


def test_norm_modulate_matches_fp64_layernorm():
    """ggml_norm restated (double sums, float steps) against an fp64
    LayerNorm; the modulate terms applied in ggml's order."""
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 1024)) * 3 + 0.5).astype(np.float32)
    s = (rng.standard_normal(1024) * 0.1).astype(np.float32)
    t = (rng.standard_normal(1024) * 0.1).astype(np.float32)
    x64 = x.astype(np.float64)
    ln = (x64 - x64.mean(1, keepdims=True)) / np.sqrt(x64.var(1, keepdims=True) + 1e-6)
    assert np.abs(O.norm_modulate(x) - ln).max() < 2e-6
    y = O.norm_modulate(x, 1e-6, s, t)
    assert np.abs(y - (ln * (1 + s) + t)).max() < 4e-6
    h = O.norm_modulate(x)
    assert np.array_equal(y, ((h * s + h) + t).astype(np.float32))   # same float steps
    assert np.array_equal(O.norm_modulate(x, 1e-6, None, t), (h + t).astype(np.float32))
    # constant rows: variance 0, output 0 (x - mean = 0; 0 / sqrt(eps))
    z = O.norm_modulate(np.full((2, 64), 3.25, np.float32))
    assert np.all(z == 0)


# ---------------------------------------------------------------- Q4_K / Q8_K
def test_q4_k_dequantizer_matches_gguf_golden():
    """Block layout and 6-bit scale/min unpacking, against gguf-py 0.19.0's
    Q4_K dequantizer (tests/golden/make_golden.py)."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "q4k_golden.npz"))
    w = g["w_q4_k"]
    assert np.array_equal(O.dequantize_q4_k(w, 512), g["w_q4_k_dequant"])


def test_q8_k_quantizer_edges():
    x = np.zeros((3, 512), np.float32)
    x[1, :256] = np.linspace(-2, 3, 256)
    x[1, 256:] = -7.0                       # constant block: iscale = -127/-7 > 0, codes -127
    x[2, 5], x[2, 9] = 4.0, -4.0            # tie in |x|: the first one sets the sign of d
    q = O.quantize_q8_k(x).reshape(3, 2, 292)
    d = q[:, :, :4].copy().view(np.float32)[:, :, 0]
    codes = q[:, :, 4:260].view(np.int8)
    bs = q[:, :, 260:].copy().view(np.int16)
    assert np.all(d[0] == 0) and np.all(codes[0] == 0) and np.all(bs[0] == 0)
    assert np.all(codes[1, 1] == -127) and d[1, 1] == np.float32(1.0) / (np.float32(-127.0) / np.float32(-7.0))
    assert codes[2, 0, 5] == -127 and codes[2, 0, 9] == 127 and d[2, 0] < 0
    assert np.array_equal(bs, codes.reshape(3, 2, 16, 16).astype(np.int32).sum(-1).astype(np.int16))
    deq = d[:, :, None] * codes.astype(np.float32)
    assert np.allclose(deq[1, 0], x[1, :256], atol=np.abs(d[1, 0]) * 0.5 + 1e-7)


def test_q4_k_dot_matches_fp64_of_dequantized():
    w = O.random_q4_k(17, 1024, 5)
    x = np.random.default_rng(6).standard_normal((9, 1024)).astype(np.float32)
    y = O.mul_mat_q4_k(w, x)
    a = O.quantize_q8_k(x).reshape(9, 4, 292)
    da = a[:, :, :4].copy().view(np.float32)[:, :, 0]
    qa = a[:, :, 4:260].view(np.int8).astype(np.float64)
    xa = (qa * da[:, :, None]).reshape(9, 1024)
    y64 = xa @ O.dequantize_q4_k(w, 1024).astype(np.float64).T
    assert rel_frobenius(y, y64) < 1e-6


def test_sparse_oracles_small_cases():
    """The scatter-mean restatement on a hand case (fp16 partial sums, zero
    start, fp32 division) and the conv restatement against an fp64 dense sum."""
    x16 = np.array([[1.0, 2048.0], [1.0, 1.0], [3.0, 1.0], [5.0, 0.5]], np.float16)
    rows = np.array([0, 0, 1, 3], np.int32)   # row 3 is outside coarse = 2: skipped
    out = O.sparse_scatter_mean_f16(x16, rows, np.array([3.0, 2.0], np.float32), 2)
    # 2048 + 1 = 2049 rounds to 2048 in fp16 (ties to even), then / 3
    assert out.tolist() == [[np.float16(2.0 / 3.0), np.float16(2048.0 / 3.0)], [1.5, 0.5]]
    rng = np.random.default_rng(0)
    t, C, cout = 20, 8, 4
    xs = rng.standard_normal((t, C)).astype(np.float16)
    w = rng.standard_normal((cout, 27 * C)).astype(np.float16)
    b = rng.standard_normal(cout).astype(np.float16)
    idx = rng.integers(-1, t, (27, t)).astype(np.int32)
    g = np.zeros((t, 27, C))
    for o in range(27):
        ok = idx[o] >= 0
        g[ok, o] = xs[idx[o][ok]]
    dense = g.reshape(t, -1) @ w.astype(np.float64).T + b
    got = O.sparse_conv_f16(xs, w, b, idx).astype(np.float64)
    assert np.max(np.abs(got - dense) / np.maximum(np.abs(dense), 1e-3)) < 2e-3
