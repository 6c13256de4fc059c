"""Symmetric peer heap: one device buffer per rank, mapped by every peer.

Each rank allocates a buffer with the same region layout (``cudaMalloc``),
exports it as a CUDA IPC handle, exchanges the handles through the process
group, and maps every peer's buffer (``cudaIpcOpenMemHandle``, peer access
over NVLink).  Kernels receive ``heaps``: a device table of every rank's
heap base in this process's address space, so ``heaps[q] + offset`` is rank
q's copy of a region.  Regions are 256-byte aligned; the last region is the
synchronization area (barrier flags and the step-statistics board).

There is no reference counterpart: the reference moves every byte through
NCCL (``minispeed/comm.py:99-141``).  The heap is what lets this library's
kernels read and write peer memory directly over NVLink.
"""

from __future__ import annotations

from typing import Dict, List, Tuple

import torch

from .. import comm
from ..ops import _ext

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
SYNC_BYTES = 4096
_ALIGN = 256


def _round(x: int) -> int:
    return -(-x // _ALIGN) * _ALIGN


class PeerHeap:
    def __init__(self, device: torch.device, regions: List[Tuple[str, int]], rank: int,
                 world: int):
        self.device = torch.device(device)
        self.rank, self.world = rank, world
        self.offsets: Dict[str, int] = {}
        self.sizes: Dict[str, int] = {}
        off = 0
        for name, nbytes in regions:
            self.offsets[name] = off
            self.sizes[name] = int(nbytes)
            off += _round(max(nbytes, 1))
        self.offsets["__sync__"] = off
        self.nbytes = off + SYNC_BYTES
        C = _ext.get()
        with torch.cuda.device(self.device):
            self.base = C.peer_alloc(self.nbytes)
            handles = comm.all_gather_object(bytes(C.peer_handle(self.base)))
            self.ptrs: List[int] = []
            self._opened: List[int] = []
            for q, h in enumerate(handles):
                if q == rank:
                    self.ptrs.append(self.base)
                else:
                    p = C.peer_open(h)
                    self._opened.append(p)
                    self.ptrs.append(p)
            self.heaps = torch.tensor(self.ptrs, dtype=torch.int64, device=self.device)
        self._closed = False

    @property
    def sync_off(self) -> int:
        return self.offsets["__sync__"]

    def view(self, name: str, dtype: torch.dtype, numel: int) -> torch.Tensor:
        """This rank's copy of region ``name`` as a tensor (heap-owned memory).
        A view larger than the region is refused: peers address the same
        layout, so an overrun would land in the next region of every rank."""
        nbytes = numel * (torch.finfo(dtype).bits // 8)
        if numel < 0 or nbytes > self.sizes[name]:
            raise ValueError(f"peer heap: {numel} x {dtype} ({nbytes} bytes) does not fit "
                             f"region {name!r} ({self.sizes[name]} bytes)")
        return _ext.get().tensor_from_ptr(self.base + self.offsets[name], numel,
                                          DTYPE_CODE[dtype], self.device.index)

    def close(self) -> None:
        if self._closed:
            return
        C = _ext.get()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for p in self._opened:
                C.peer_close(p)
            C.peer_free(self.base)
        self._closed = True
