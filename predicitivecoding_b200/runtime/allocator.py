"""Python face of the native stream-ordered caching allocator (C++ in the extension).

Reference: PredictiveCoding.Device/Allocators/CudaAllocator.cs:19-104 (cudaMalloc per tensor,
cudaFree on dispose, byte counters).  ``alloc`` returns a torch tensor whose storage goes back to
the native cache when the tensor dies; nothing is returned to the driver until ``empty_cache``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .. import ops

_ELT = {torch.float32: 4, torch.bfloat16: 2, torch.float16: 2, torch.int32: 4, torch.int64: 8, torch.uint8: 1,
        torch.int8: 1}


@dataclass(frozen=True)
class AllocatorStats:
    allocated: int
    reserved: int
    peak: int
    allocations: int
    cache_hits: int
    driver_allocations: int


class DeviceAllocator:
    def __init__(self, device: int = 0):
        self.device = device

    def alloc(self, shape, dtype=torch.float32, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        shape = tuple(shape) if not isinstance(shape, int) else (shape,)
        n = 1
        for s in shape:
            n *= s
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        raw = ops.ext().dev_alloc(max(1, n * _ELT[dtype]), self.device, st)
        return raw[: n * _ELT[dtype]].view(dtype).view(shape)

    def zeros(self, shape, dtype=torch.float32, stream=None) -> torch.Tensor:
        return self.alloc(shape, dtype, stream).zero_()

    def record_stream(self, t: torch.Tensor, stream: torch.cuda.Stream) -> None:
        ops.ext().dev_record_stream(t, stream.cuda_stream)

    def stats(self) -> AllocatorStats:
        return AllocatorStats(*ops.ext().dev_alloc_stats(self.device))

    def reset_peak(self) -> None:
        ops.ext().dev_alloc_reset_peak(self.device)

    def empty_cache(self) -> None:
        ops.ext().dev_release_cached(self.device)


CANARY_BYTES = 256
_CANARY_BYTE = 0xA5


class CanaryAllocator(DeviceAllocator):
    """Debug allocator: every block gets CANARY_BYTES of a fixed byte pattern behind it; `verify()`
    reports blocks whose guard was overwritten (an out-of-bounds write by some kernel)."""

    def __init__(self, device: int = 0):
        super().__init__(device)
        self._blocks = []

    def alloc(self, shape, dtype=torch.float32, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
        shape = tuple(shape) if not isinstance(shape, int) else (shape,)
        n = 1
        for s in shape:
            n *= s
        nbytes = max(1, n * _ELT[dtype])
        st = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        raw = ops.ext().dev_alloc(nbytes + CANARY_BYTES, self.device, st)
        raw[nbytes:nbytes + CANARY_BYTES].fill_(_CANARY_BYTE)
        self._blocks.append((raw, nbytes))
        return raw[:nbytes].view(dtype).view(shape)

    def verify(self) -> list:
        """Indices of blocks whose guard bytes changed (synchronises the device)."""
        torch.cuda.synchronize(self.device)
        return [i for i, (raw, n) in enumerate(self._blocks)
                if not bool((raw[n:n + CANARY_BYTES] == _CANARY_BYTE).all())]
