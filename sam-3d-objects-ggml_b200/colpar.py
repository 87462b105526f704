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
    """One device buffer per rank, every rank holding device addresses of all
    of them (its own plus CUDA-IPC mappings of the peers'): fp32 [rows][cols]
    by default, or `nbytes` bytes (a prepared-activation buffer)."""

    def __init__(self, rows: int, cols: int, group=None, nbytes: int | None = None):
        import torch.distributed as dist
        from cuda.bindings import runtime as cudart

        import torch

        self._cudart = cudart
        _ok(cudart.cudaSetDevice(torch.cuda.current_device())[0], "cudaSetDevice")
        self.rows, self.cols = rows, cols
        self.nbytes = rows * cols * 4 if nbytes is None else nbytes
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
        """Copy of this rank's buffer as a torch tensor (fp32 [rows][cols], or
        uint8 [nbytes] for a byte-sized buffer)."""
        import torch
        if self.nbytes != self.rows * self.cols * 4:
            t = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        else:
            t = torch.empty((self.rows, self.cols), dtype=torch.float32, device=device)
        err, = self._cudart.cudaMemcpy(t.data_ptr(), self.local, self.nbytes,
                                       self._cudart.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
        _ok(err, "cudaMemcpy")
        return t

    def local_tensor(self, device):
        """This rank's buffer as a uint8 torch tensor sharing its memory (no
        copy), e.g. as the next GEMM's operand; valid until close()."""
        import torch
        ptr, nbytes = self.local, self.nbytes

        class _Mem:
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                        "version": 3, "strides": None}
        return torch.as_tensor(_Mem(), device=device)

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


def activation_buffers(m: int, n_total: int, group=None) -> PeerBuffers:
    """Every rank's prepared Q8_0 activation buffer for [m][n_total] (the next
    layer's input), mapped on every rank."""
    return PeerBuffers(m, n_total, group=group, nbytes=b2q.act_prepared_size(m, n_total))


def fused_gelu_q8(packed_slice, n_slice: int, k: int, act, m: int, abufs: PeerBuffers, col0: int, bias=None,
                  stream=None) -> None:
    """This rank's rows [col0, col0 + n_slice) through GELU + Q8_0 straight into
    every rank's next-layer activations (launch only): the exchange is 1.125
    bytes per value instead of fp32's 4."""
    b2q.mul_mat_prepared_gelu_q8_peers(packed_slice, n_slice, k, act, m, abufs.ptrs, abufs.cols, col0,
                                       abufs.nbytes, bias=bias, stream=stream)


def split_views(buf, m: int, n: int):
    """(codes [m][n] int8, scales [n/32][ld] fp32) views of a prepared Q8_0
    activation buffer (uint8 tensor) in the library's split layout."""
    import torch
    ld = (m + 3) // 4 * 4
    codes_bytes = (m * n + 255) // 256 * 256
    codes = buf[:m * n].view(torch.int8).view(m, n)
    scales = buf[codes_bytes:codes_bytes + (n // 32) * ld * 4].view(torch.float32).view(n // 32, ld)
    return codes, scales


def nccl_baseline_gelu_q8(packed_slice, n_slice: int, k: int, act, m: int, n_total: int, local, gathered_codes,
                          gathered_scales, out, bias=None, group=None, stream=None):
    """GELU + Q8_0 into this rank's [m][n_slice] activations, NCCL all-gather of
    the codes and of the scales, codes transposed into [m][n_total] (equal
    slices only): the same bytes cross the links as the fused form."""
    import torch.distributed as dist
    b2q.mul_mat_prepared_gelu_q8(packed_slice, n_slice, k, act, m, bias=bias, out=local, stream=stream)
    lc, ls = split_views(local, m, n_slice)
    oc, osc = split_views(out, m, n_total)
    dist.all_gather_into_tensor(gathered_codes, lc, group=group)
    dist.all_gather_into_tensor(gathered_scales, ls, group=group)
    world = gathered_codes.shape[0] // m
    oc.copy_(gathered_codes.view(world, m, n_slice).permute(1, 0, 2).reshape(m, n_total))
    osc.copy_(gathered_scales.view(n_total // 32, ls.shape[1]))
    return out


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


__all__ = ["slices", "PeerBuffers", "fused", "nccl_baseline", "activation_buffers", "fused_gelu_q8",
           "split_views", "nccl_baseline_gelu_q8"]
