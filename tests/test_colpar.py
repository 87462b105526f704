"""Column-parallel mul_mat (b2q_mul_mat_prepared_peers) and its Q8_0-exchange
form (b2q_mul_mat_prepared_gelu_q8_peers): each rank holds a slice of the
weight's output rows and its GEMM epilogue writes the slice into every rank's
full-width output -- fp32, or the next layer's prepared Q8_0 activations --
over peer memory.  The GPU cases need two GPUs of one box (they are skipped
otherwise); the slice plan and the entry's argument checks run on CPU."""
import os
import socket
import time

import numpy as np
import pytest

import colpar

RTOL = 1e-5  # relative Frobenius tolerance of the fp32 result


@pytest.mark.parametrize("n_total,world", [(3072, 8), (3072, 2), (200, 2), (1000, 3), (33, 4), (0, 2)])
def test_slices_cover_rows_in_32_row_units(n_total, world):
    sl = colpar.slices(n_total, world)
    assert len(sl) == world
    assert sl[0][0] == 0 and sl[-1][1] == n_total
    for (a, b), (c, _) in zip(sl, sl[1:]):
        assert b == c and a <= b
    for a, b in sl:
        assert a % 32 == 0 or a == b  # empty slices sit at the end
        assert (b - a) % 32 == 0 or b == n_total
    units = [(b - a + 31) // 32 for a, b in sl]  # 32-row units per rank differ by at most one
    assert max(units) - min(units) <= 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, M, N, K, wtype):
    import datetime
    import torch
    import torch.distributed as dist
    import b2q
    import oracle as O
    from helpers import make_case, rel_frobenius

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        _, wq, x = make_case(M + N + K, M, N, K, wtype)  # same seed on every rank
        bias = np.random.default_rng(N).standard_normal(N).astype(np.float32)
        w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
        x_d = torch.from_numpy(x).to(dev)
        b_d = torch.from_numpy(bias).to(dev)
        start, stop = colpar.slices(N, world)[rank]
        packed = b2q.weight_pack(wtype, w_d[start:stop], K)
        act = b2q.act_prepare(x_d)
        bufs = colpar.PeerBuffers(M, N)
        bufs.fill_nan()
        torch.cuda.synchronize()
        dist.barrier()
        colpar.fused(packed, stop - start, K, act, M, bufs, start, bias=b_d[start:stop])
        torch.cuda.synchronize()
        dist.barrier()  # every rank's kernel has finished writing every buffer
        got = bufs.to_tensor(dev)
        full = b2q.mul_mat(wtype, w_d, x_d, bias=b_d)
        torch.cuda.synchronize()
        assert torch.equal(got, full), "column-parallel result differs from the single-GPU GEMM"
        if rank == 0:
            ref = O.mul_mat(wtype, wq, x, O.ACT_X86) + bias[None, :]
            assert rel_frobenius(got.cpu().numpy(), ref) <= RTOL
        assert b2q.device_status(clear=True) == 0
        dist.barrier()
        bufs.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,wtype", [(300, 256, 512, 2), (129, 200, 1024, 8), (1024, 3072, 1024, 2)])
def test_fused_column_parallel_matches_single_gpu(b2q_mod, M, N, K, wtype):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one box")
    world = 2
    ctx = mp.start_processes(_rank_main, args=(world, _free_port(), M, N, K, wtype), nprocs=world,
                             join=False, start_method="spawn")
    deadline = time.time() + 240
    try:
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                raise TimeoutError("column-parallel ranks did not finish")
    finally:
        for p in ctx.processes:
            if p.is_alive():
                p.kill()


def _rank_main_q8(rank, world, port, M, N, K, wtype):
    import datetime
    import torch
    import torch.distributed as dist
    import b2q
    from helpers import make_case

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        _, wq, x = make_case(M + N + K + 1, M, N, K, wtype)  # same seed on every rank
        bias = np.random.default_rng(N + 1).standard_normal(N).astype(np.float32)
        w_d = torch.from_numpy(np.ascontiguousarray(wq)).to(dev)
        b_d = torch.from_numpy(bias).to(dev)
        start, stop = colpar.slices(N, world)[rank]
        n = stop - start
        full_packed = b2q.weight_pack(wtype, w_d, K)
        packed = b2q.weight_pack(wtype, w_d[start:stop], K)
        act = b2q.act_prepare(torch.from_numpy(x).to(dev))
        abufs = colpar.activation_buffers(M, N)
        torch.cuda.synchronize()
        dist.barrier()
        colpar.fused_gelu_q8(packed, n, K, act, M, abufs, start, bias=b_d[start:stop])
        torch.cuda.synchronize()
        dist.barrier()  # every rank's kernel has finished writing every buffer
        got = abufs.to_tensor(dev)
        want = b2q.mul_mat_prepared_gelu_q8(full_packed, N, K, act, M, bias=b_d)
        torch.cuda.synchronize()
        gc, gs = colpar.split_views(got, M, N)
        wc, ws = colpar.split_views(want, M, N)
        assert torch.equal(gc, wc), "Q8_0 codes differ from the single-GPU GELU + Q8_0 epilogue"
        assert torch.equal(gs[:, :M], ws[:, :M]), "Q8_0 scales differ from the single-GPU epilogue"
        # the NCCL baseline moves the same bytes to the same places
        local = b2q._empty_aligned(b2q.act_prepared_size(M, n), dev)
        gcodes = torch.empty((world * M, n), dtype=torch.int8, device=dev)
        ld = (M + 3) // 4 * 4
        gscales = torch.empty((world * (n // 32), ld), dtype=torch.float32, device=dev)
        out = b2q._empty_aligned(b2q.act_prepared_size(M, N), dev)
        colpar.nccl_baseline_gelu_q8(packed, n, K, act, M, N, local, gcodes, gscales, out, bias=b_d[start:stop])
        torch.cuda.synchronize()
        oc, osc = colpar.split_views(out, M, N)
        assert torch.equal(oc, wc) and torch.equal(osc[:, :M], ws[:, :M])
        assert b2q.device_status(clear=True) == 0
        dist.barrier()
        abufs.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,wtype", [(300, 256, 512, 2), (129, 1024, 1024, 8), (2048, 4096, 1024, 2)])
def test_q8_exchange_column_parallel_matches_single_gpu(b2q_mod, M, N, K, wtype):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one box")
    world = 2
    ctx = mp.start_processes(_rank_main_q8, args=(world, _free_port(), M, N, K, wtype), nprocs=world,
                             join=False, start_method="spawn")
    deadline = time.time() + 240
    try:
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                raise TimeoutError("column-parallel ranks did not finish")
    finally:
        for p in ctx.processes:
            if p.is_alive():
                p.kill()


INVALID_ARG = 1


@pytest.mark.parametrize("n,n_total,col0,expect", [
    (64, 256, 16, INVALID_ARG),   # col0 not a whole Q8_0 block
    (48, 256, 0, INVALID_ARG),    # slice not a whole number of blocks
    (64, 100, 64, INVALID_ARG),   # next-layer K not a whole number of blocks
    (128, 192, 128, INVALID_ARG),  # slice runs past the next-layer K
])
def test_q8_exchange_rejects_bad_slices(b2q_mod, n, n_total, col0, expect):
    import ctypes
    lib = b2q_mod.lib()
    arr = (ctypes.c_void_p * 1)(256)
    rc = lib.b2q_mul_mat_prepared_gelu_q8_peers(256, n, 64, 256, 8, None, arr, 1, n_total, col0, 1 << 20,
                                                b2q_mod.ACT_X86, None)
    assert rc == expect


def test_q8_exchange_rejects_too_many_peers(b2q_mod):
    import ctypes
    lib = b2q_mod.lib()
    arr = (ctypes.c_void_p * 9)(*([256] * 9))
    rc = lib.b2q_mul_mat_prepared_gelu_q8_peers(256, 64, 64, 256, 8, None, arr, 9, 256, 0, 1 << 20,
                                                b2q_mod.ACT_X86, None)
    assert rc == INVALID_ARG


@pytest.mark.parametrize("m,n", [(1, 32), (129, 1024), (300, 256), (20480, 4096)])
def test_split_views_match_the_library_layout(b2q_mod, m, n):
    """colpar.split_views (the NCCL baseline's view of a prepared-activation
    buffer) against the library's own size arithmetic: codes [m][n] at 0,
    scales [n/32][round_up(m, 4)] fp32 at the next 256-byte boundary."""
    import torch
    size = b2q_mod.act_prepared_size(m, n)
    buf = torch.zeros(size, dtype=torch.uint8)
    codes, scales = colpar.split_views(buf, m, n)
    ld = (m + 3) // 4 * 4
    assert codes.shape == (m, n) and scales.shape == (n // 32, ld)
    assert codes.data_ptr() == buf.data_ptr()
    off = scales.data_ptr() - buf.data_ptr()
    assert off == (m * n + 255) // 256 * 256
    assert off + scales.numel() * 4 <= size
    assert size == off + ((n // 32) * ld * 4 + 255) // 256 * 256


def _rank_main_mlp(rank, world, port, M, C, H):
    import datetime
    import torch
    import torch.distributed as dist
    import b2q
    from helpers import make_case

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        _, w1, x = make_case(11, M, H, C, 2)
        _, w2, _ = make_case(12, 1, C, H, 2)
        b1 = torch.from_numpy(np.random.default_rng(3).standard_normal(H).astype(np.float32)).to(dev)
        b2 = torch.from_numpy(np.random.default_rng(4).standard_normal(C).astype(np.float32)).to(dev)
        s1, e1 = colpar.slices(H, world)[rank]
        s2, e2 = colpar.slices(C, world)[rank]
        p1 = b2q.weight_pack(2, torch.from_numpy(w1[s1:e1]).to(dev), C)
        p2 = b2q.weight_pack(2, torch.from_numpy(w2[s2:e2]).to(dev), H)
        act = b2q.act_prepare(torch.from_numpy(x).to(dev))
        hid = colpar.activation_buffers(M, H)
        ybuf = colpar.PeerBuffers(M, C)
        hid_t = hid.local_tensor(dev)
        torch.cuda.synchronize()
        dist.barrier()
        colpar.fused_gelu_q8(p1, e1 - s1, C, act, M, hid, s1, bias=b1[s1:e1])
        torch.cuda.synchronize()
        dist.barrier()  # every rank's fc1 slice is in every rank's fc2 input
        colpar.fused(p2, e2 - s2, H, hid_t, M, ybuf, s2, bias=b2[s2:e2])
        torch.cuda.synchronize()
        dist.barrier()
        got = ybuf.to_tensor(dev)
        h_ref = b2q.mul_mat_prepared_gelu_q8(b2q.weight_pack(2, torch.from_numpy(w1).to(dev), C), H, C, act, M,
                                             bias=b1)
        y_ref = b2q.mul_mat_prepared(b2q.weight_pack(2, torch.from_numpy(w2).to(dev), H), C, H, h_ref, M, bias=b2)
        torch.cuda.synchronize()
        assert torch.equal(got, y_ref), "sharded MLP differs from the single-GPU MLP"
        assert b2q.device_status(clear=True) == 0
        dist.barrier()
        del hid_t
        hid.close()
        ybuf.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("M,C,H", [(300, 256, 1024), (1000, 1024, 4096)])
def test_sharded_mlp_matches_single_gpu(b2q_mod, M, C, H):
    """fc1 column-parallel with the Q8_0 exchange, then fc2 column-parallel with
    the fp32 gather: every rank ends with the single-GPU MLP's output, bit for bit."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs of one box")
    world = 2
    ctx = mp.start_processes(_rank_main_mlp, args=(world, _free_port(), M, C, H), nprocs=world, join=False,
                             start_method="spawn")
    deadline = time.time() + 240
    try:
        while not ctx.join(timeout=5):
            if time.time() > deadline:
                raise TimeoutError("sharded MLP ranks did not finish")
    finally:
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
