"""Peer-memory group: symmetric device buffers shared between the ranks of one node.

Each rank allocates the same-sized buffer with ``cudaMalloc`` and exports a CUDA
IPC handle; handles are exchanged once through ``torch.distributed`` and every
rank opens its peers' buffers.  The result is a device table of ``world``
pointers per buffer that fused kernels (``rs_adamw_ag``, ``pc_allreduce_update``,
``peer_reduce``) use to load and store peer memory directly over NVLink /
NVSwitch.  The reference has no device collectives at all: its NCCL provider is
a host-side mock (PredictiveCoding.Device/Nccl/NcclProvider.cs:1-109).

No multicast object is created and no TMA is ever pointed at a peer buffer: the
kernels use plain loads and stores.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import ops

_ELT = {torch.float32: 4, torch.bfloat16: 2, torch.int32: 4, torch.uint8: 1, torch.int64: 8, torch.float64: 8}


@dataclass
class SymmetricBuffer:
    local: torch.Tensor        # this rank's buffer (typed view)
    ptrs: torch.Tensor         # device int64 [world]: every rank's buffer address, as seen from this rank
    host_ptrs: List[int]       # the same addresses on the host (for copy-engine transfers)


class PeerGroup:
    """All ranks of ``pg`` on one node, with IPC-mapped symmetric buffers and a device barrier."""

    def __init__(self, pg=None, device: Optional[torch.device] = None):
        self.pg = pg
        self.world = dist.get_world_size(pg) if dist.is_initialized() else 1
        self.rank = dist.get_rank(pg) if dist.is_initialized() else 0
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        if self.device.index is None:   # "cuda" means the current device
            self.device = torch.device("cuda", torch.cuda.current_device())
        self._opened: List[int] = []
        self._keep: List[torch.Tensor] = []
        self.flags = self.symmetric(64, torch.int32)
        self.ctr = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)

    def symmetric(self, numel: int, dtype: torch.dtype) -> SymmetricBuffer:
        nbytes = ((numel * _ELT[dtype] + 255) // 256) * 256
        raw = ops.ext().peer_alloc(nbytes, self.device.index)
        self._keep.append(raw)
        handle = ops.ext().ipc_handle(raw)
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=self.pg)
        else:
            handles = [handle]
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(raw.data_ptr())
            else:
                p = ops.ext().ipc_open(h)
                self._opened.append(p)
                ptrs.append(p)
        table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        local = raw.view(dtype)[:numel]
        return SymmetricBuffer(local, table, ptrs)

    def barrier(self) -> None:
        """Device-side barrier over all ranks, ordered on the current stream (bounded wait)."""
        ops.ext().peer_barrier(self.flags.ptrs, self.ctr, self.rank, self.world, self.err)

    def check(self) -> None:
        """Raise if any bounded wait in a peer kernel timed out."""
        code = int(self.err.item())
        if code:
            raise RuntimeError(f"peer collective timed out on rank {self.rank} (error code {code})")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            ops.ext().ipc_close(p)
        self._opened.clear()
        self._keep.clear()
