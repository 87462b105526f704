"""The SLat sparse stages on the device against the oracle's restatement of
the reference's CPU operators (ggml patch 0001-sam3d-ggml-combined.patch:
151-272): the F16 scatter-mean (2x downsample), bit-exact; the F16
submanifold convolution (gather of the 27 neighbour rows + kind::f16 GEMM),
within one fp16 rounding step of the CPU's fp32-accumulated result plus the
worst-case fp32 summation error of the two orders (the tensor core sums in a
different order; both results are rounded to fp16), and equal in >= 97% of the
outputs."""
import numpy as np
import pytest

import b2q
import oracle as O

pytestmark = pytest.mark.gpu


def to_dev(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.fixture(autouse=True)
def _no_device_errors(b2q_mod, dev):
    yield
    assert b2q.device_status(clear=True) == 0


def sparse_grid(grid: int, occupancy: float, seed: int):
    """Active cells sampled without replacement, their 27-neighbour table
    (offset-major, -1 = missing) and the 2x-downsample mapping."""
    rng = np.random.default_rng(seed)
    n = int(round(occupancy * grid ** 3))
    keys = np.sort(rng.choice(grid ** 3, n, replace=False))
    xyz = np.stack([keys // (grid * grid), (keys // grid) % grid, keys % grid], 1)
    idx = np.full((27, n), -1, np.int32)
    o = 0
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                q = xyz + np.array([dx, dy, dz])
                inside = np.all((q >= 0) & (q < grid), 1)
                qk = (q[:, 0] * grid + q[:, 1]) * grid + q[:, 2]
                pos = np.clip(np.searchsorted(keys, qk), 0, n - 1)
                hit = inside & (keys[pos] == qk)
                idx[o, hit] = pos[hit]
                o += 1
    ck = ((xyz[:, 0] // 2) * (grid // 2) + xyz[:, 1] // 2) * (grid // 2) + xyz[:, 2] // 2
    coarse_keys, rows = np.unique(ck, return_inverse=True)
    counts = (np.bincount(rows, minlength=coarse_keys.size) + 1).astype(np.float32)  # + the initial zero row
    return idx, rows.astype(np.int32), counts, coarse_keys.size


@pytest.mark.parametrize("C", [8, 128])
def test_scatter_mean_bit_exact_on_a_downsample(dev, C):
    _, rows, counts, coarse = sparse_grid(40, 0.03, 1)
    rng = np.random.default_rng(C)
    x16 = (rng.standard_normal((rows.size, C)) * 3).astype(np.float16)
    got = b2q.sparse_scatter_mean_f16(to_dev(x16, dev), to_dev(rows, dev), to_dev(counts, dev), coarse)
    want = O.sparse_scatter_mean_f16(x16, rows, counts, coarse)
    assert np.array_equal(got.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_scatter_mean_order_fanin_skips_and_overflow(dev):
    """Large fan-in (order of the fp16 partial sums matters), rows outside the
    coarse range skipped, empty coarse rows, sums that overflow fp16."""
    C, coarse, fine = 16, 37, 3000
    rng = np.random.default_rng(4)
    rows = rng.integers(-2, coarse + 2, fine).astype(np.int32)
    rows[rows == 5] = 6                                   # coarse row 5 stays empty
    x16 = (rng.standard_normal((fine, C)) * 50).astype(np.float16)
    x16[rows == 7] = np.float16(30000)                    # row 7 saturates to inf
    counts = (rng.integers(1, 9, coarse)).astype(np.float32)
    got = b2q.sparse_scatter_mean_f16(to_dev(x16, dev), to_dev(rows, dev), to_dev(counts, dev), coarse)
    want = O.sparse_scatter_mean_f16(x16, rows, counts, coarse)
    g = got.cpu().numpy()
    assert np.array_equal(g.view(np.uint16), want.view(np.uint16))
    assert np.all(g[5] == 0) and np.all(np.isinf(g[7]))
    # a second call on the same workspace-free path gives the same bytes
    again = b2q.sparse_scatter_mean_f16(to_dev(x16, dev), to_dev(rows, dev), to_dev(counts, dev), coarse)
    assert np.array_equal(again.cpu().numpy().view(np.uint16), want.view(np.uint16))


def test_scatter_plan_reused_across_calls(dev):
    """One plan serves several feature sets (the mapping is fixed per object):
    the planned accumulation equals the one-shot operator bit for bit."""
    _, rows, counts, coarse = sparse_grid(32, 0.04, 7)
    rows_d, counts_d = to_dev(rows, dev), to_dev(counts, dev)
    plan = b2q.sparse_scatter_plan(rows_d, coarse)
    rng = np.random.default_rng(9)
    for _ in range(2):
        x16 = (rng.standard_normal((rows.size, 64)) * 2).astype(np.float16)
        got = b2q.sparse_scatter_mean_f16_planned(to_dev(x16, dev), plan, counts_d, coarse)
        want = O.sparse_scatter_mean_f16(x16, rows, counts, coarse)
        assert np.array_equal(got.cpu().numpy().view(np.uint16), want.view(np.uint16))


def _conv_bound(x16, w16, idx, want):
    """Largest allowed |GPU - CPU| per output: one fp16 step of the CPU value
    (both round their fp32 sum to fp16) plus twice the worst-case fp32
    summation error of either order, K * 2^-24 * sum |w * x| (K = 27 * C)."""
    tokens, C = x16.shape
    g = np.zeros((tokens, 27, C))
    for o in range(27):
        ok = (idx[o] >= 0) & (idx[o] < tokens)
        g[ok, o] = np.abs(x16[idx[o][ok]].astype(np.float64))
    s = g.reshape(tokens, -1) @ np.abs(w16.astype(np.float64)).T
    step = np.spacing(np.abs(want).astype(np.float16)).astype(np.float64)
    return step + 2.0 * 27 * C * 2.0 ** -24 * s


@pytest.mark.parametrize("C,cout,bias", [(8, 128, True), (64, 96, False), (128, 128, True)])
def test_sparse_conv_matches_cpu_operator(dev, C, cout, bias):
    idx, _, _, _ = sparse_grid(24, 0.05, C)
    tokens = idx.shape[1]
    rng = np.random.default_rng(C + cout)
    x16 = rng.standard_normal((tokens, C)).astype(np.float16)
    w16 = (rng.standard_normal((cout, 27 * C)) / np.sqrt(27 * C)).astype(np.float16)
    b16 = (rng.standard_normal(cout) * 0.1).astype(np.float16) if bias else None
    got = b2q.sparse_conv_f16(to_dev(x16, dev), to_dev(w16, dev), to_dev(b16, dev) if bias else None,
                              to_dev(idx, dev)).cpu().numpy()
    want = O.sparse_conv_f16(x16, w16, b16, idx)
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(np.isfinite(got))
    assert np.all(err <= _conv_bound(x16, w16, idx, want))
    assert np.mean(err == 0) >= 0.97            # almost always the same fp16 value


def test_sparse_conv_missing_neighbours_and_out_of_range(dev):
    """A token whose neighbours are all missing returns its bias; indices >=
    tokens count as missing, like -1."""
    C, cout, tokens = 16, 32, 50
    rng = np.random.default_rng(2)
    x16 = rng.standard_normal((tokens, C)).astype(np.float16)
    w16 = (rng.standard_normal((cout, 27 * C)) * 0.1).astype(np.float16)
    b16 = rng.standard_normal(cout).astype(np.float16)
    idx = rng.integers(-1, tokens + 3, (27, tokens)).astype(np.int32)
    idx[:, 0] = -1
    idx[:, 1] = tokens + 1
    got = b2q.sparse_conv_f16(to_dev(x16, dev), to_dev(w16, dev), to_dev(b16, dev), to_dev(idx, dev)).cpu().numpy()
    want = O.sparse_conv_f16(x16, w16, b16, idx)
    assert np.array_equal(got[0], b16) and np.array_equal(got[1], b16)
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= _conv_bound(x16, w16, idx, want))


@pytest.mark.parametrize("grid,occ,C,cout,bias", [(24, 0.05, 64, 96, True), (20, 0.3, 128, 128, False),
                                                  (16, 0.02, 256, 64, True)])
def test_planned_conv_matches_cpu_operator(dev, grid, occ, C, cout, bias):
    """The planned convolution (only occupied neighbour pairs, grouped GEMM,
    ordered fp32 reduce) against the CPU operator, with the same bound as the
    dense form, and one plan reused for two inputs."""
    idx, _, _, _ = sparse_grid(grid, occ, C + cout)
    tokens = idx.shape[1]
    rng = np.random.default_rng(C * 3 + cout)
    w16 = (rng.standard_normal((cout, 27 * C)) / np.sqrt(27 * C)).astype(np.float16)
    b16 = (rng.standard_normal(cout) * 0.1).astype(np.float16) if bias else None
    idx_d = to_dev(idx, dev)
    plan = b2q.sparse_conv_plan(idx_d)
    for _ in range(2):
        x16 = rng.standard_normal((tokens, C)).astype(np.float16)
        got = b2q.sparse_conv_f16_planned(to_dev(x16, dev), to_dev(w16, dev), to_dev(b16, dev) if bias else None,
                                          plan).cpu().numpy()
        want = O.sparse_conv_f16(x16, w16, b16, idx)
        err = np.abs(got.astype(np.float64) - want.astype(np.float64))
        assert np.all(np.isfinite(got))
        assert np.all(err <= _conv_bound(x16, w16, idx, want))
        assert np.mean(err == 0) >= 0.97


def test_planned_conv_isolated_tokens_and_out_of_range(dev):
    """Tokens with no valid neighbour return the bias; indices >= tokens are
    missing; a table with every slot empty gives the bias everywhere."""
    C, cout, tokens = 64, 32, 300
    rng = np.random.default_rng(12)
    x16 = rng.standard_normal((tokens, C)).astype(np.float16)
    w16 = (rng.standard_normal((cout, 27 * C)) * 0.05).astype(np.float16)
    b16 = rng.standard_normal(cout).astype(np.float16)
    idx = np.where(rng.random((27, tokens)) < 0.1, rng.integers(0, tokens + 5, (27, tokens)), -1).astype(np.int32)
    idx[:, :3] = -1
    got = b2q.sparse_conv_f16_planned(to_dev(x16, dev), to_dev(w16, dev), to_dev(b16, dev),
                                      b2q.sparse_conv_plan(to_dev(idx, dev))).cpu().numpy()
    want = O.sparse_conv_f16(x16, w16, b16, idx)
    assert np.array_equal(got[:3], np.tile(b16, (3, 1)))
    err = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.all(err <= _conv_bound(x16, w16, idx, want))
    empty = np.full((27, tokens), -1, np.int32)
    got = b2q.sparse_conv_f16_planned(to_dev(x16, dev), to_dev(w16, dev), to_dev(b16, dev),
                                      b2q.sparse_conv_plan(to_dev(empty, dev))).cpu().numpy()
    assert np.array_equal(got, np.tile(b16, (tokens, 1)))
