"""Column-parallel mul_mat over the GPUs of one box (host side).

For a single large mul_mat (the SLat flow transformer's linears at 8k-20k
tokens) the weight is split by output rows across the ranks of a group and
every rank needs the whole [M][N] output afterwards.  Two ways to run it:

* fused (the product): each rank runs ``b2q_mul_mat_prepared_peers`` on its
  weight rows; the GEMM epilogue stores every finished tile straight into all
  ranks' full-width output buffers over NVLink (P2P stores into CUDA-IPC mapped
  peer memory), so the gather overlaps the remaining tiles' math and no
  transpose is needed;
* nccl (the baseline): each rank computes its [M][N/P] slice, then
  ``all_gather_into_tensor`` and a [P][M][N/P] -> [M][N] transpose.

One process per GPU, ``torch.distributed`` with the NCCL backend for the
plumbing (handle exchange, barriers, the baseline's all-gather).  Peer buffers
are plain ``cudaMalloc`` allocations shared with CUDA IPC: no multicast
objects, no symmetric-memory layer.
"""
from __future__ import annotations

import b2q


def slices(n_total: int, world: int) -> list[tuple[int, int]]:
    """Weight-row ranges [start, stop) per rank: contiguous, as even as
    possible, each a multiple of 32 rows except the last (so no rank's slice
    starts inside another rank's 32-row TMEM quarter)."""
    if world < 1 or n_total < 0:
        raise ValueError("world >= 1 and n_total >= 0 required")
    unit = 32
    units = (n_total + unit - 1) // unit
    out, start = [], 0
    for r in range(world):
        take = units // world + (1 if r < units % world else 0)
        stop = min(n_total, start + take * unit)
        out.append((start, stop))
        start = stop
    return out


class PeerBuffers:
    """One fp32 [rows][cols] buffer per rank, every rank holding device
    addresses of all of them (its own plus CUDA-IPC mappings of the peers')."""

    def __init__(self, rows: int, cols: int, group=None):
        import torch.distributed as dist
        from cuda.bindings import runtime as cudart

        import torch

        self._cudart = cudart
        _ok(cudart.cudaSetDevice(torch.cuda.current_device())[0], "cudaSetDevice")
        self.rows, self.cols = rows, cols
        self.nbytes = rows * cols * 4
        single = not (dist.is_available() and dist.is_initialized())
        self.rank, self.world = (0, 1) if single else (dist.get_rank(group), dist.get_world_size(group))
        err, ptr = cudart.cudaMalloc(self.nbytes)
        _ok(err, "cudaMalloc")
        self.local = int(ptr)
        err, handle = cudart.cudaIpcGetMemHandle(ptr)
        _ok(err, "cudaIpcGetMemHandle")
        handles = [bytes(handle.reserved)]
        if not single:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.reserved), group=group)
        self.ptrs, self._opened = [], []
        for r, hb in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.local)
                continue
            h = cudart.cudaIpcMemHandle_t()
            h.reserved = hb
            err, p = cudart.cudaIpcOpenMemHandle(h, cudart.cudaIpcMemLazyEnablePeerAccess)
            _ok(err, "cudaIpcOpenMemHandle")
            self.ptrs.append(int(p))
            self._opened.append(p)

    def fill_nan(self) -> None:
        err, = self._cudart.cudaMemset(self.local, 0xFF, self.nbytes)  # 0xFFFFFFFF is a NaN
        _ok(err, "cudaMemset")

    def to_tensor(self, device):
        """Copy of this rank's buffer as a torch tensor."""
        import torch
        t = torch.empty((self.rows, self.cols), dtype=torch.float32, device=device)
        err, = self._cudart.cudaMemcpy(t.data_ptr(), self.local, self.nbytes,
                                       self._cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
        _ok(err, "cudaMemcpy")
        return t

    def close(self) -> None:
        for p in self._opened:
            self._cudart.cudaIpcCloseMemHandle(p)
        self._opened = []
        if self.local:
            self._cudart.cudaFree(self.local)
            self.local = 0


def _ok(err, what: str) -> None:
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: {err}")


def fused(packed_slice, n_slice: int, k: int, act, m: int, bufs: PeerBuffers, col0: int, bias=None,
          stream=None) -> None:
    """This rank's rows [col0, col0 + n_slice) into every rank's buffer (launch only)."""
    b2q.mul_mat_prepared_peers(packed_slice, n_slice, k, act, m, bufs.ptrs, col0, bufs.cols * 4,
                               bias=bias, stream=stream)


def nccl_baseline(packed_slice, n_slice: int, k: int, act, m: int, n_total: int, slice_out, gathered, out,
                  group=None, stream=None):
    """GEMM on this rank's rows, NCCL all-gather of the [M][n] slices, transpose
    into [M][N] (equal slices only)."""
    import torch.distributed as dist
    b2q.mul_mat_prepared(packed_slice, n_slice, k, act, m, out=slice_out, stream=stream)
    dist.all_gather_into_tensor(gathered, slice_out, group=group)
    world = gathered.shape[0] // m
    out.copy_(gathered.view(world, m, n_slice).permute(1, 0, 2).reshape(m, n_total))
    return out


__all__ = ["slices", "PeerBuffers", "fused", "nccl_baseline"]
