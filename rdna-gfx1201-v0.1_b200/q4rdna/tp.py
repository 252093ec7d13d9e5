"""Tensor-parallel row sharding of Q4_RDNA tensors (one process per GPU).

Rank r of P owns output rows [r*N/P, (r+1)*N/P) of every tensor and computes
them from the replicated activation x.  A 32-row band of the tile stream is one
contiguous run of (K/64)*1088 bytes (tile (row_tile, group) sits at
(row_tile*G + group)*1088, the order written by the reference packers,
q4rdna_sidecar_pack.cpp:268-278), so the shard of a packed tensor is a byte
slice of it and sharding needs no repacking.  Shards are whole 32-row bands, so
N must be a multiple of 32*P.

Each rank concatenates the y slices of all its tensors into one buffer (the
order of the tensor list).  One all-gather of those buffers leaves every rank
with all outputs, rank-major; `Layout.assemble` puts the pieces back per tensor.
Rows are independent, so the assembled y of every tensor equals, bit for bit,
the y a single GPU computes with the same split factor.
"""

from __future__ import annotations

from dataclasses import dataclass

TILE_ROWS = 32
GROUP = 64
TILE_BYTES = 1088


def shard_rows(N: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of rank `rank`'s shard of an N-row tensor."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if N % (TILE_ROWS * world):
        raise ValueError(f"{N} rows do not split into {world} shards of whole 32-row bands")
    rows = N // world
    return rank * rows, rows


def shard_tiles(tiles, N: int, K: int, world: int, rank: int):
    """Rank `rank`'s rows of a packed N x K tensor: a slice (no copy) of the
    1-D uint8 tile stream `tiles` (numpy array or torch tensor)."""
    if K % GROUP:
        raise ValueError("K % 64 must be 0")
    band = (K // GROUP) * TILE_BYTES
    if tiles.shape[0] != (N // TILE_ROWS) * band:
        raise ValueError(f"tile stream holds {tiles.shape[0]} bytes, {N}x{K} needs {(N // TILE_ROWS) * band}")
    row0, rows = shard_rows(N, world, rank)
    b0 = (row0 // TILE_ROWS) * band
    return tiles[b0:b0 + (rows // TILE_ROWS) * band]


@dataclass(frozen=True)
class Slot:
    name: str
    N: int        # full rows
    K: int
    rows: int     # rows per rank
    offset: int   # start of this tensor's slice in a rank's y buffer, in rows (x B floats)


class Layout:
    """Where every tensor's y slice sits in a rank's y buffer, and how the
    gathered buffers map back to full outputs.

    A rank's y buffer holds B * ysz f32: tensor i's slice is the contiguous
    [B][rows_i] block at float B * offset_i, the y layout the kernels write
    (y[b * N + n]).  The gathered buffer is [world][B * ysz].
    """

    def __init__(self, tensors, world: int, B: int = 1):
        self.world, self.B = world, B
        self.slots: list[Slot] = []
        off = 0
        for (name, N, K) in tensors:
            _, rows = shard_rows(N, world, 0)
            self.slots.append(Slot(name, N, K, rows, off))
            off += rows
        self.ysz = off
        self.xsz = sum(s.K for s in self.slots)

    def __len__(self):
        return len(self.slots)

    def local_view(self, y_rank, i: int):
        """Tensor i's slice of a rank's y buffer, shaped [B, rows] (a view)."""
        s = self.slots[i]
        B = self.B
        return y_rank.reshape(-1)[B * s.offset:B * (s.offset + s.rows)].reshape(B, s.rows)

    def assemble(self, gathered) -> list:
        """Full outputs [B, N] per tensor from the gathered [world][B * ysz]
        buffer (numpy or torch; the result has the same type)."""
        B = self.B
        g = gathered.reshape(self.world, B * self.ysz)
        out = []
        for s in self.slots:
            parts = [g[r, B * s.offset:B * (s.offset + s.rows)].reshape(B, s.rows) for r in range(self.world)]
            out.append(_cat(parts))
        return out


def _cat(parts):
    if hasattr(parts[0], "cpu"):  # torch
        import torch

        return torch.cat(parts, dim=1)
    import numpy as np

    return np.concatenate(parts, axis=1)


def all_gather(y_rank, gathered, group=None) -> None:
    """Gather every rank's y buffer into `gathered` ([world * numel] f32, rank
    order) with torch.distributed: one NCCL all-gather on GPU ranks, the list
    form on gloo."""
    import torch.distributed as dist

    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, y_rank, group=group)
        return
    world = dist.get_world_size(group)
    parts = list(gathered.view(world, -1).unbind(0))
    dist.all_gather(parts, y_rank.reshape(-1), group=group)


class _DeviceBuffer:
    """Exposes library-owned device memory to torch (no copy)."""

    def __init__(self, ptr: int, nfloats: int):
        self.__cuda_array_interface__ = {"shape": (nfloats,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


class PeerGather:
    """The all-gather fused into the plan kernel (q4rdna_plan_set_gather).

    Every rank allocates two gathered buffers (world x its y buffer) and one
    flag array in IPC-shareable device memory, exchanges the handles over the
    process group and maps its peers' buffers.  Each plan run then stores every
    output also into this rank's slice of every rank's gathered buffer (plain
    NVLink peer stores from the GEMV epilogue) and ends with a bounded flag
    exchange, so that when the run's work on this GPU has finished, the
    gathered buffer it returns holds every rank's outputs of that run.  Runs
    alternate between the two buffers, so a rank running one step ahead never
    overwrites a buffer a slower rank is still reading.
    """

    def __init__(self, plan, layout: Layout, y_rank, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib, check

        lib = _lib()
        self._lib = lib
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        if y_rank.numel() != layout.B * layout.ysz:
            raise ValueError("y buffer does not match the layout")
        self.world, self.rank, self.plan = world, rank, plan
        nrank = layout.B * layout.ysz
        sizes = [4 * world * nrank, 4 * world * nrank, 256]
        self._own, handles = [], []
        for nb in sizes:
            ptr, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            check(lib.q4rdna_ipc_alloc(nb, ctypes.byref(ptr), h), "ipc_alloc")
            self._own.append(ptr.value)
            handles.append(h.raw)
        allh = [None] * world
        dist.all_gather_object(allh, handles, group=group)
        self._opened = []
        maps = [[0] * world for _ in sizes]
        for p in range(world):
            for k in range(len(sizes)):
                if p == rank:
                    maps[k][p] = self._own[k]
                    continue
                ptr = ctypes.c_void_p()
                check(lib.q4rdna_ipc_open(allh[p][k], ctypes.byref(ptr)), "ipc_open")
                self._opened.append(ptr.value)
                maps[k][p] = ptr.value
        arr = [(ctypes.c_void_p * world)(*m) for m in maps]
        check(lib.q4rdna_plan_set_gather(plan._h, world, rank, y_rank.data_ptr(), nrank, arr[0], arr[1], arr[2]),
              "plan_set_gather")
        dev = y_rank.device
        self.gathered = [torch.as_tensor(_DeviceBuffer(self._own[k], world * nrank), device=dev) for k in (0, 1)]
        # every rank has mapped every buffer before any rank's first run
        dist.barrier(group=group)

    def run(self, stream=None):
        """One plan run with its fused gather; returns the gathered buffer
        ([world * B * ysz] f32, rank-major) that the run fills."""
        self.plan.run(stream)
        return self.gathered[self._lib.q4rdna_plan_gather_parity(self.plan._h)]

    def close(self):
        """Unmap the peers' buffers and free this rank's.  Every rank must have
        finished its runs (the caller synchronises and barriers first)."""
        import torch.distributed as dist

        for p in self._opened:
            self._lib.q4rdna_ipc_close(p)
        self._opened = []
        self.gathered = []
        dist.barrier()  # peers have unmapped this rank's buffers
        for p in self._own:
            self._lib.q4rdna_ipc_free(p)
        self._own = []
