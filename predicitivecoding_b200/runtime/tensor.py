"""Device tensors and the op dispatch used by the device-side examples and serving helpers.

Reference: PredictiveCoding.Device/DeviceTensor.cs:20-142 (FromHost / To / ToHost / EmptyLike,
shape, device id, stream) and TensorOps.cs:17-104 (MatMul through the GEMM provider, CopyTo,
Synchronize).  On a GPU the storage comes from the native caching allocator, ``matmul`` runs the
tcgen05 GEMM, the row ops run the extension's kernels; on the CPU the same calls run in torch.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

from .. import ops
from .allocator import DeviceAllocator
from .device import Device, DeviceRuntime


class DeviceTensor:
    def __init__(self, data: torch.Tensor, device: Device):
        self.data = data
        self.device = device
        self.stream = None

    @staticmethod
    def from_host(host, device: Optional[Device] = None) -> "DeviceTensor":
        t = torch.as_tensor(host)
        dev = DeviceRuntime.resolve(device or Device.cpu())
        if dev.is_cpu:
            return DeviceTensor(t.clone(), dev)
        out = DeviceAllocator(dev.id).alloc(t.shape, t.dtype)
        out.copy_(t, non_blocking=False)
        return DeviceTensor(out, dev)

    @staticmethod
    def zeros(shape: Sequence[int], dtype=torch.float32, device: Optional[Device] = None) -> "DeviceTensor":
        dev = DeviceRuntime.resolve(device or Device.cpu())
        if dev.is_cpu:
            return DeviceTensor(torch.zeros(tuple(shape), dtype=dtype), dev)
        return DeviceTensor(DeviceAllocator(dev.id).zeros(tuple(shape), dtype), dev)

    def to(self, target: Device) -> "DeviceTensor":
        target = DeviceRuntime.resolve(target)
        if target == self.device:
            return self
        return DeviceTensor.from_host(self.to_host(), target)

    def to_host(self) -> torch.Tensor:
        return self.data.detach().cpu().clone()

    def empty_like(self) -> "DeviceTensor":
        return DeviceTensor.zeros(self.shape, self.data.dtype, self.device)

    @property
    def shape(self):
        return tuple(self.data.shape)

    @property
    def element_count(self) -> int:
        return self.data.numel()

    @property
    def size_in_bytes(self) -> int:
        return self.data.numel() * self.data.element_size()

    @property
    def is_on_device(self) -> bool:
        return self.device.is_gpu


class TensorOps:
    @staticmethod
    def matmul(a: DeviceTensor, b: DeviceTensor) -> DeviceTensor:
        """C[m, n] = A[m, k] @ B[k, n]; fp32 result.  GPU: tcgen05 GEMM on bf16 operands."""
        if a.shape[1] != b.shape[0]:
            raise ValueError(f"inner dimensions differ: {a.shape} @ {b.shape}")
        if a.device.is_cpu:
            return DeviceTensor(a.data.float() @ b.data.float(), a.device)
        k, n = a.shape[1], b.shape[1]
        if k % 8 == 0 and n % 8 == 0:
            c = ops.gemm(a.data.to(torch.bfloat16).contiguous(), b.data.to(torch.bfloat16).contiguous(), b_mn=True,
                         epi=ops.EPI_F32)
        else:
            c = a.data.float() @ b.data.float()
        return DeviceTensor(c, a.device)

    @staticmethod
    def copy_to(src: DeviceTensor, dst: DeviceTensor) -> None:
        dst.data.copy_(src.data)

    @staticmethod
    def softmax_rows(x: DeviceTensor, scale: float = 1.0) -> DeviceTensor:
        if x.device.is_cpu:
            return DeviceTensor(torch.softmax(x.data.float() * scale, -1), x.device)
        return DeviceTensor(ops.softmax_rows(x.data.float().contiguous(), scale), x.device)

    @staticmethod
    def gelu(x: DeviceTensor) -> DeviceTensor:
        return DeviceTensor(torch.nn.functional.gelu(x.data, approximate="tanh"), x.device)

    @staticmethod
    def add_(dst: DeviceTensor, src: DeviceTensor) -> None:
        dst.data.add_(src.data)

    @staticmethod
    def scale_(x: DeviceTensor, alpha: float) -> None:
        x.data.mul_(alpha)

    @staticmethod
    def synchronize(stream=None) -> None:
        if torch.cuda.is_available():
            (stream or torch.cuda.current_stream()).synchronize()
