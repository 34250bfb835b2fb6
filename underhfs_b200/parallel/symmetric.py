"""Symmetric device memory shared by all ranks of a node.

Each rank allocates one region with the native ``SymmetricHeap`` (device
memory exported through CUDA IPC), the IPC handles are exchanged once over
the torch.distributed process group, and every rank maps every peer's region.
Tensors carved out of the local region are ordinary torch tensors (DLPack,
no copy); the fused collective kernels address the same offsets on every peer.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from underhfs_b200.ops._lib import core


class SymmetricBuffer:
    def __init__(self, nbytes: int, *, rank: int, world: int, group=None) -> None:
        c = core()
        self.rank = rank
        self.world = world
        self.heap = c.SymmetricHeap(rank, world, int(nbytes))
        handle = self.heap.ipc_handle()
        if world > 1:
            handles: list = [None] * world
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        self.heap.open(handles)
        self.nbytes = int(self.heap.data_bytes)
        self._cursor = 0
        self._views: list[torch.Tensor] = []

    def tensor(self, numel: int, dtype: torch.dtype, *, offset_bytes: int | None = None) -> torch.Tensor:
        """A 1-D view of the local region; by default carved sequentially
        (256-byte aligned) so every rank gets identical offsets."""
        esize = torch.empty((), dtype=dtype).element_size()
        if offset_bytes is None:
            offset_bytes = (self._cursor + 255) // 256 * 256
            self._cursor = offset_bytes + numel * esize
        if offset_bytes + numel * esize > self.nbytes:
            raise MemoryError("symmetric buffer exhausted")
        name = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.int32: "int32",
                torch.uint8: "uint8"}[dtype]
        t = torch.utils.dlpack.from_dlpack(self.heap.dlpack(offset_bytes, numel, name))
        t._uhfs_sym = self  # keep the heap alive as long as the view
        t._uhfs_offset = offset_bytes
        self._views.append(t)
        return t

    @staticmethod
    def offset_of(t: torch.Tensor) -> int:
        base = getattr(t, "_uhfs_offset", None)
        if base is not None:
            return base
        raise ValueError("tensor is not a view of a symmetric buffer")

    def close(self) -> None:
        self.heap.close()
