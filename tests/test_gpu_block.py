"""GPU check of one SS-flow DiT block (sam-3d-objects-ggml_b200/ss_block.py)
against its CPU composition from the oracle (reference_forward), and of the
attention I/O kernels (b2q_qkv_heads, b2q_heads_act_prepare) on their own.

Bars: the fp16 q, k, v equal their CPU restatement bit for bit except where the
fp32 RMS scale's last bit differs (< 0.1% of values, one fp16 step); the Q8_0
output-projection activations equal act_prepare of the same fp32 values bit for
bit; the whole block within BLOCK_RTOL of the CPU composition (the attention
core runs in fp16 through a library kernel, and every mul_mat's 1e-5 passes
through the next quantize)."""
import numpy as np
import pytest

import b2q
import oracle as O

pytestmark = pytest.mark.gpu

BLOCK_RTOL = 2e-3


def to_dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.fixture(autouse=True)
def _no_device_errors(b2q_mod, dev):
    yield
    assert b2q.device_status(clear=True) == 0


@pytest.mark.parametrize("H", [4, 5])  # even H: the float4 kernel; odd H: the 32-lane kernel
def test_qkv_heads_matches_cpu(dev, H):
    import torch
    B, T, D = 2, 37, 64
    C = H * D
    rng = np.random.default_rng(1)
    qkv = (rng.standard_normal((B * T, 3 * C + 8)) * 2).astype(np.float32)   # padded rows
    gq = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    gk = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    d = to_dev(qkv, dev)
    q, k, v = b2q.qkv_heads(d[:, :3 * C], B, T, H, D, to_dev(gq, dev), to_dev(gk, dev))
    torch.cuda.synchronize()

    def ref(t, g):
        t = t.reshape(B, T, H, D)
        if g is None:
            return t.astype(np.float16).transpose(0, 2, 1, 3)
        ms = ((t.astype(np.float64) ** 2).sum(-1, keepdims=True) / D).astype(np.float32)
        sc = np.float32(1.0) / np.sqrt(ms + np.float32(1e-6))
        return ((t * sc) * g.reshape(H, D)).astype(np.float16).transpose(0, 2, 1, 3)

    for got, want in ((q, ref(qkv[:, :C], gq)), (k, ref(qkv[:, C:2 * C], gk)), (v, ref(qkv[:, 2 * C:3 * C], None))):
        g = got.cpu().numpy()
        diff = g.astype(np.float32) != want.astype(np.float32)
        assert diff.mean() < 1e-3
        assert np.all(np.abs(g.astype(np.float32) - want.astype(np.float32)) <= np.abs(np.spacing(want)).astype(np.float32) + 1e-12)


@pytest.mark.parametrize("parts", [1, 2])
@pytest.mark.parametrize("D", [32, 64])
def test_rows_to_heads_is_fp16_transpose(dev, parts, D):
    """The cross-attention's q (parts 1) and k | v (parts 2) rows -> fp16
    heads: a plain round-to-nearest conversion and a transpose, bit-exact
    (D = 64 takes the two-heads-per-warp float4 kernel)."""
    B, T, H = 2, 45, 8
    C = H * D
    rng = np.random.default_rng(7 + parts)
    rows = (rng.standard_normal((B * T, parts * C + 4)) * 3).astype(np.float32)
    outs = b2q.rows_to_heads(to_dev(rows, dev)[:, :parts * C], B, T, H, D, parts)
    assert len(outs) == parts
    for p, got in enumerate(outs):
        want = rows[:, p * C:(p + 1) * C].reshape(B, T, H, D).astype(np.float16).transpose(0, 2, 1, 3)
        assert tuple(got.shape) == (B, H, T, D)
        assert np.array_equal(got.cpu().numpy().view(np.uint16), np.ascontiguousarray(want).view(np.uint16))


@pytest.mark.parametrize("parts,B,T,H,wtype", [(1, 2, 300, 16, O.TYPE_Q8_0),   # cross q: token tiles cross a sequence
                                                (2, 2, 1374, 16, O.TYPE_Q8_0),  # k | v of the condition tokens
                                                (2, 1, 45, 4, O.TYPE_Q4_0),     # one sequence, ragged last tile
                                                (1, 3, 9, 2, O.TYPE_Q8_0)])     # sequences shorter than a tile
def test_mul_mat_heads_equals_two_steps(dev, parts, B, T, H, wtype):
    """The projection's tile end writing fp16 heads: the same bytes as
    mul_mat_prepared (+ bias) followed by rows_to_heads, with and without a bias."""
    import torch
    D, K = 64, 256
    N, M = parts * H * D, B * T
    rng = np.random.default_rng(100 + parts * T)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float32)
    packed = b2q.weight_pack(wtype, to_dev(O.quantize(w, wtype), dev), K)
    act = b2q.act_prepare(to_dev(x, dev))
    for bb in (None, to_dev(bias, dev)):
        y = b2q.mul_mat_prepared(packed, N, K, act, M, bias=bb)
        want = b2q.rows_to_heads(y, B, T, H, D, parts)
        got = b2q.mul_mat_prepared_heads(packed, N, K, act, B, T, H, D, bias=bb)
        torch.cuda.synchronize()
        assert len(got) == parts
        for g, wnt in zip(got, want):
            assert tuple(g.shape) == (B, H, T, D)
            assert np.array_equal(g.cpu().numpy().view(np.uint16), wnt.cpu().numpy().view(np.uint16))


@pytest.mark.parametrize("variant", [0, 1])
def test_layer_norm_q8_matches_oracle(dev, variant):
    """gb_layer_norm (ggml_norm, * weight, + bias) with the Q8_0 quantize of
    the next mul_mat fused in: the same bytes as the oracle's."""
    M, C = 300, 1024
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((M, C)) * 2).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    bb = (0.1 * rng.standard_normal(C)).astype(np.float32)
    act = b2q.layer_norm_q8(to_dev(x, dev), 1e-6, to_dev(w, dev), to_dev(bb, dev), variant=variant)
    a = act.cpu().numpy()
    h = O.norm_modulate(x, 1e-6) * w + bb
    ref = O.quantize(h.astype(np.float32), O.TYPE_Q8_0, variant).reshape(M, C // 32, 34)
    assert np.array_equal(a[:M * C].view(np.int8).reshape(M, C // 32, 32), ref[:, :, 2:].view(np.int8))
    off, ld = (M * C + 255) // 256 * 256, (M + 3) // 4 * 4
    sc = a[off:off + (C // 32) * ld * 4].view(np.float32).reshape(C // 32, ld)[:, :M]
    d16 = ref[:, :, :2].copy().view(np.float16).reshape(M, C // 32).astype(np.float32)
    assert np.array_equal(sc.T, d16 * np.float32(2.0 ** 49))


def test_heads_act_prepare_equals_act_prepare(dev):
    import torch
    B, T, H, D = 2, 50, 4, 64
    o = torch.randn(B, T, H, D, device=dev).half().permute(0, 2, 1, 3)   # [B, H, T, D] view, t-major memory
    act = b2q.heads_act_prepare(o)
    rows = o.permute(0, 2, 1, 3).reshape(B * T, H * D).float().contiguous()
    ref = b2q.act_prepare(rows)
    torch.cuda.synchronize()
    M, K = B * T, H * D
    a, r = act.cpu().numpy(), ref.cpu().numpy()
    off, ld = (M * K + 255) // 256 * 256, (M + 3) // 4 * 4
    assert np.array_equal(a[:M * K], r[:M * K])
    sa = a[off:off + (K // 32) * ld * 4].view(np.float32).reshape(K // 32, ld)[:, :M]
    sr = r[off:off + (K // 32) * ld * 4].view(np.float32).reshape(K // 32, ld)[:, :M]
    assert np.array_equal(sa.view(np.uint32), sr.view(np.uint32))


def reference_forward(blk, x, B: int, T: int, cond, n_cond: int):
    """The block on the CPU from the oracle's ggml restatements (norm, quantized
    mul_mat, GELU) and an fp64 softmax attention on the fp16-rounded q, k, v."""
    v = {k: t.cpu().numpy() for k, t in blk.vec.items()}
    C, H, D, wt = blk.C, blk.H, blk.D, blk.wtype
    h = O.norm_modulate(x, 1e-6, v["scale_msa"], v["shift_msa"])
    qkv = O.mul_mat(wt, blk.raw["qkv"], h, O.ACT_X86) + v["b_qkv"]

    def heads(t, g):
        t = t.reshape(B, T, H, D).astype(np.float32)
        if g is not None:
            ms = ((t.astype(np.float64) ** 2).sum(-1, keepdims=True) / D).astype(np.float32)
            t = (t * (np.float32(1.0) / np.sqrt(ms + np.float32(1e-6)))) * g.reshape(H, D)
        return t.astype(np.float16).astype(np.float64).transpose(0, 2, 1, 3)  # [B, H, T, D]

    def attend(q, k, vv):
        s = q @ k.transpose(0, 1, 3, 2) / np.sqrt(D)
        # the flash kernel's P operand is fp16; its row sum adds those fp16 values
        s = np.exp(s - s.max(-1, keepdims=True)).astype(np.float16).astype(np.float64)
        o = (s @ vv) / s.sum(-1, keepdims=True)
        return o.astype(np.float16).astype(np.float32).transpose(0, 2, 1, 3).reshape(-1, C)

    q, k, vv = heads(qkv[:, :C], v["gq"]), heads(qkv[:, C:2 * C], v["gk"]), heads(qkv[:, 2 * C:], None)
    o = attend(q, k, vv)
    x = x + (O.mul_mat(wt, blk.raw["out"], o, O.ACT_X86) + v["b_out"]) * v["gate_msa"]
    # cross-attention: affine LayerNorm, q from x, k | v from cond, residual without gate
    h = O.norm_modulate(x) * v["n2w"] + v["n2b"]
    xq = O.mul_mat(wt, blk.raw["xq"], h, O.ACT_X86) + v["b_xq"]
    xkv = O.mul_mat(wt, blk.raw["xkv"], cond, O.ACT_X86) + v["b_xkv"]
    ch = lambda t, n: t.reshape(B, n, H, D).astype(np.float16).astype(np.float64).transpose(0, 2, 1, 3)  # noqa: E731
    o = attend(ch(xq, T), ch(xkv[:, :C], n_cond), ch(xkv[:, C:], n_cond))
    x = x + (O.mul_mat(wt, blk.raw["xout"], o, O.ACT_X86) + v["b_xout"])
    h = O.norm_modulate(x, 1e-6, v["scale_mlp"], v["shift_mlp"])
    h = O.gelu(O.mul_mat(wt, blk.raw["fc1"], h, O.ACT_X86) + v["b1"])
    return x + (O.mul_mat(wt, blk.raw["fc2"], h, O.ACT_X86) + v["b2"]) * v["gate_mlp"]


@pytest.mark.parametrize("wtype", [O.TYPE_Q8_0, O.TYPE_Q4_0])
def test_ss_block_matches_cpu_composition(dev, wtype):
    import torch
    import ss_block
    B, T, C, H = 2, 128, 256, 4
    rng = np.random.default_rng(3)
    weights = {name: O.quantize((rng.standard_normal(sh) * 0.02).astype(np.float32), wtype)
               for name, sh in ss_block.SsBlock.shapes(C, 4 * C).items()}
    blk = ss_block.SsBlock(dev, weights, C=C, heads=H, wtype=wtype, seed=3)
    x = np.random.default_rng(4).standard_normal((B * T, C)).astype(np.float32)
    n_cond = 77
    cond = np.random.default_rng(5).standard_normal((B * n_cond, C)).astype(np.float32)
    xd = to_dev(x, dev)
    blk.forward(xd, B, T, to_dev(cond, dev), n_cond)
    torch.cuda.synchronize()
    y = xd.cpu().numpy()
    ref = reference_forward(blk, x, B, T, cond, n_cond)
    err = np.linalg.norm((y - ref).astype(np.float64)) / np.linalg.norm(ref.astype(np.float64))
    assert err <= BLOCK_RTOL, err
