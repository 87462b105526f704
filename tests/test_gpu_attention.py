"""The tensor-core attention core (b2q_attention_f16, gb_attention's production
flash path with F16 K/V, cpp_ggml/src/graph_builder.cpp:151-171) against an fp64
softmax of the same fp16 inputs, at the SS-flow shapes (self-attention over
4096 tokens, cross-attention to 1374 condition tokens, the 4-token pose group
over its own and the shape keys) and ragged ones.  The kernel rounds P and o to
fp16 as the flash path does, so the bar is a few fp16 steps; torch's SDPA on the
same inputs is measured beside it as a yardstick."""
import math

import numpy as np
import pytest

import b2q

RTOL = 2e-3  # relative Frobenius vs fp64: fp16 rounding of P and of o


def ref_f64(q, k, v, k2=None, v2=None):
    q, k, v = (a.double() for a in (q, k, v))
    if k2 is not None:
        import torch
        k, v = torch.cat([k, k2.double()], 2), torch.cat([v, v2.double()], 2)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    o = s.softmax(-1) @ v
    B, H, Tq, D = o.shape
    return o.permute(0, 2, 1, 3).reshape(B * Tq, H * D)


def rel(a, b):
    return float((a.double() - b).norm() / b.norm())


@pytest.mark.gpu
@pytest.mark.parametrize("B,H,Tq,Tk,Tk2", [
    (2, 16, 4096, 4096, 0),   # SS self-attention
    (2, 16, 4096, 1374, 0),   # SS cross-attention
    (2, 16, 4, 4, 4096),      # pose group: its own keys, then the shape keys
    (1, 2, 100, 70, 0),       # ragged query and key tiles
    (1, 3, 1, 129, 5),        # one query; a key tile of one; second source of five
])
def test_attention_f16_matches_fp64(b2q_mod, dev, B, H, Tq, Tk, Tk2):
    import torch
    g = torch.Generator(device=dev).manual_seed(B * 100 + Tq + Tk + Tk2)
    mk = lambda t: (torch.randn(B, H, t, 64, device=dev, generator=g) * 1.5).half()  # noqa: E731
    q, k, v = mk(Tq), mk(Tk), mk(Tk)
    k2 = v2 = None
    if Tk2:
        k2, v2 = mk(Tk2), mk(Tk2)
    o = b2q.attention_f16(q, k, v, k2, v2)
    ref = ref_f64(q, k, v, k2, v2)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all()
    err = rel(o, ref)
    kk = k if k2 is None else torch.cat([k, k2], 2)
    vv = v if v2 is None else torch.cat([v, v2], 2)
    sdpa = torch.nn.functional.scaled_dot_product_attention(q, kk, vv).permute(0, 2, 1, 3).reshape(B * Tq, H * 64)
    assert err <= RTOL, f"rel {err:.2e} (torch SDPA on the same inputs: {rel(sdpa, ref):.2e})"
    assert b2q.device_status() == 0


@pytest.mark.gpu
def test_attention_f16_output_feeds_the_projection_quantizer(b2q_mod, dev):
    """The row layout is what b2q_heads_act_prepare reads with strides: the
    prepared activations equal those of the same values in [B, H, T, D] form."""
    import torch
    B, H, T = 2, 16, 300
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v = ((torch.randn(B, H, T, 64, device=dev, generator=g)).half() for _ in range(3))
    o_rows = b2q.attention_f16(q, k, v)                         # [B*T, H*64]
    o_bhtd = o_rows.view(B, T, H, 64).permute(0, 2, 1, 3)        # strided view
    a = b2q.heads_act_prepare(o_bhtd)
    b = b2q.heads_act_prepare(o_bhtd.contiguous())
    assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [0, 1])
@pytest.mark.parametrize("B,H,Tq,Tk,Tk2", [
    (2, 16, 4096, 4096, 0),   # SS self-attention
    (2, 16, 4096, 1374, 0),   # SS cross-attention
    (2, 16, 4, 4, 4096),      # pose group: its own keys, then the shape keys
    (1, 2, 100, 70, 0),       # ragged query and key tiles
    (3, 3, 257, 129, 5),      # a partial second query tile; second source of five
])
def test_attention_f16_q8_equals_attention_then_quantize(b2q_mod, dev, variant, B, H, Tq, Tk, Tk2):
    """The fused Q8_0 output writes the bytes of heads_act_prepare applied to
    attention_f16's fp16 rows, codes and split scales alike."""
    import torch
    g = torch.Generator(device=dev).manual_seed(B * 1000 + Tq + Tk + Tk2 + variant)
    q = torch.randn(B, H, Tq, 64, device=dev, generator=g).half()
    k, v = (torch.randn(B, H, Tk, 64, device=dev, generator=g).half() for _ in range(2))
    k2 = v2 = None
    if Tk2:
        k2, v2 = (torch.randn(B, H, Tk2, 64, device=dev, generator=g).half() for _ in range(2))
    o = b2q.attention_f16(q, k, v, k2, v2).view(B, Tq, H, 64).permute(0, 2, 1, 3)
    ref = b2q.heads_act_prepare(o, variant=variant)
    got = b2q.attention_f16_q8(q, k, v, k2, v2, variant=variant)
    torch.cuda.synchronize()
    M, K = B * Tq, H * 64
    mp = (M + 3) // 4 * 4
    code_bytes = M * K
    scale_off = (code_bytes + 255) // 256 * 256
    assert torch.equal(got[:code_bytes], ref[:code_bytes])
    gs = got[scale_off:scale_off + 4 * mp * (K // 32)].view(torch.float32).view(K // 32, mp)[:, :M]
    rs = ref[scale_off:scale_off + 4 * mp * (K // 32)].view(torch.float32).view(K // 32, mp)[:, :M]
    assert torch.equal(gs, rs)
    assert b2q.device_status() == 0


FAKE = 1 << 20


@pytest.mark.parametrize("args,expect", [
    ((FAKE, FAKE, FAKE, 1, 2, 64, 64, 32, None, None, 0, 0.125, 0, FAKE, 1 << 20), 2),   # D != 64: unsupported
    ((FAKE, FAKE, FAKE, 1, 2, 64, 64, 64, None, None, 0, 0.125, 7, FAKE, 1 << 20), 1),   # variant
    ((FAKE, FAKE, FAKE, 1, 2, 64, 64, 64, FAKE, None, 4, 0.125, 0, FAKE, 1 << 20), 1),   # k2 without v2
    ((FAKE, FAKE, FAKE, 1, 2, 64, 64, 64, None, None, 0, 0.125, 0, FAKE + 16, 1 << 20), 3),  # act alignment
    ((FAKE, FAKE, FAKE, 1, 2, 64, 64, 64, None, None, 0, 0.125, 0, FAKE, 100), 4),       # act too small
])
def test_attention_f16_q8_argument_checks(b2q_mod, args, expect):
    assert b2q_mod.lib().b2q_attention_f16_q8(*args, None) == expect
