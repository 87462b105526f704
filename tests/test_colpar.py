"""Column-parallel mul_mat (b2q_mul_mat_prepared_peers): each rank holds a slice
of the weight's output rows and its GEMM epilogue writes the slice into every
rank's full-width output over peer memory.  The GPU case needs two GPUs of one
box (it is skipped otherwise); the slice plan is checked on CPU."""
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
