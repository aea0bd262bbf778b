"""Devices, their resolution and the process-wide default.

Reference: PredictiveCoding.Device/Device.cs:11-39 (Cpu / Cuda(id) / CudaMulti / Metal / Rocm),
DeviceRuntime.cs:14-83 (device counts, ``Resolve`` maps CudaMulti to device 0 and unavailable
GPUs to the CPU) and DeviceRegistry.cs:14-67 (EnableCuda / UseCpu / AutoSelect).  This build targets
one vendor: Metal and ROCm are accepted as names and always resolve to the CPU.  ``CudaMulti``
resolves to this process's GPU (``LOCAL_RANK``), one process per GPU.
"""
from __future__ import annotations

import enum
import os
from dataclasses import dataclass

import torch


class DeviceKind(enum.Enum):
    CPU = "cpu"
    CUDA = "cuda"
    CUDA_MULTI = "cudamulti"
    METAL = "metal"
    ROCM = "rocm"


@dataclass(frozen=True)
class Device:
    kind: DeviceKind
    id: int = 0

    @staticmethod
    def cpu() -> "Device":
        return Device(DeviceKind.CPU)

    @staticmethod
    def cuda(id: int = 0) -> "Device":
        return Device(DeviceKind.CUDA, id)

    @staticmethod
    def cuda_multi() -> "Device":
        return Device(DeviceKind.CUDA_MULTI)

    @staticmethod
    def metal(id: int = 0) -> "Device":
        return Device(DeviceKind.METAL, id)

    @staticmethod
    def rocm(id: int = 0) -> "Device":
        return Device(DeviceKind.ROCM, id)

    @property
    def is_cpu(self) -> bool:
        return self.kind == DeviceKind.CPU

    @property
    def is_gpu(self) -> bool:
        return not self.is_cpu

    @property
    def is_cuda(self) -> bool:
        return self.kind in (DeviceKind.CUDA, DeviceKind.CUDA_MULTI)

    def __str__(self) -> str:
        return "cpu" if self.is_cpu else f"{self.kind.value}:{self.id}"

    def torch(self) -> torch.device:
        return DeviceRuntime.resolve(self).torch_device()

    def torch_device(self) -> torch.device:
        return torch.device("cpu") if self.is_cpu else torch.device("cuda", self.id)


class DeviceRuntime:
    @staticmethod
    def cuda_device_count() -> int:
        try:
            return torch.cuda.device_count() if torch.cuda.is_available() else 0
        except Exception:
            return 0

    @staticmethod
    def cuda_available() -> bool:
        return DeviceRuntime.cuda_device_count() > 0

    @staticmethod
    def multi_gpu_available() -> bool:
        return DeviceRuntime.cuda_device_count() > 1

    @staticmethod
    def native_loaded() -> bool:
        try:
            from .. import ops
            ops.ext()
            return True
        except Exception:
            return False

    @staticmethod
    def resolve(requested: Device) -> Device:
        n = DeviceRuntime.cuda_device_count()
        if requested.kind == DeviceKind.CUDA_MULTI:
            if n == 0:
                return Device.cpu()
            return Device.cuda(int(os.environ.get("LOCAL_RANK", "0")) % n)
        if requested.kind == DeviceKind.CUDA:
            return requested if requested.id < n else Device.cpu()
        return Device.cpu()


class DeviceRegistry:
    cuda_enabled = False
    _current = None

    @classmethod
    def default_device(cls) -> Device:
        if cls._current is not None:
            return cls._current
        return Device.cuda(0) if DeviceRuntime.cuda_available() else Device.cpu()

    @classmethod
    def enable_cuda(cls, device_id: int = 0) -> bool:
        if device_id < DeviceRuntime.cuda_device_count():
            cls.cuda_enabled = True
            cls._current = Device.cuda(device_id)
            torch.cuda.set_device(device_id)
            return True
        return False

    @classmethod
    def enable_rocm(cls, device_id: int = 0) -> bool:
        return False

    @classmethod
    def use_cpu(cls) -> None:
        cls.cuda_enabled = False
        cls._current = Device.cpu()

    @classmethod
    def auto_select(cls) -> Device:
        if cls.enable_cuda(int(os.environ.get("LOCAL_RANK", "0")) % max(1, DeviceRuntime.cuda_device_count())):
            return cls._current
        cls.use_cpu()
        return cls._current
