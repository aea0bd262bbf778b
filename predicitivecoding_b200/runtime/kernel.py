"""Runtime-compiled CUDA kernels: CUDA C source -> NVRTC (sm_100a cubin) -> module -> launches.

Reference: PredictiveCoding.Device/Kernels/CudaKernel.cs:1-125 (NVRTC compile to PTX, cuModuleLoadData,
cuModuleGetFunction, synchronous Launch1D/Launch and asynchronous *OnStream variants, argument
marshalling, primary-context retain).  Here NVRTC emits a cubin for the exact target (no PTX JIT at load
time), the module is loaded into the context PyTorch already made current, and arguments are marshalled
from torch tensors (device pointers), Python ints (int32 unless wrapped) and floats (float32).
The framework's own hot kernels are compiled ahead of time into the extension; this is the plug point
for user kernels, as the reference's CudaKernel is for its NVRTC strings.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple, Union

import numpy as np
import torch


class KernelCompileError(RuntimeError):
    pass


@dataclass(frozen=True)
class I64:
    """Marks a Python int that the kernel takes as a 64-bit integer."""
    value: int


def _check_nvrtc(err, prog=None, what=""):
    from cuda.bindings import nvrtc
    if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        log = ""
        if prog is not None:
            _, n = nvrtc.nvrtcGetProgramLogSize(prog)
            buf = b" " * n
            nvrtc.nvrtcGetProgramLog(prog, buf)
            log = buf.decode(errors="replace")
        raise KernelCompileError(f"{what}: {err}\n{log}")


def compile_cubin(source: str, name: str = "kernel.cu", arch: str = "sm_100a",
                  options: Sequence[str] = ()) -> bytes:
    """Compile CUDA C source with NVRTC for one architecture; returns the cubin bytes (no GPU needed)."""
    from cuda.bindings import nvrtc
    err, prog = nvrtc.nvrtcCreateProgram(source.encode(), name.encode(), 0, [], [])
    if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        raise KernelCompileError(f"nvrtcCreateProgram: {err}")
    try:
        opts = [f"--gpu-architecture={arch}".encode(), b"-default-device", b"-std=c++17"] + [o.encode() for o in options]
        err, = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
        _check_nvrtc(err, prog, "nvrtcCompileProgram")
        err, size = nvrtc.nvrtcGetCUBINSize(prog)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            raise KernelCompileError(f"nvrtcGetCUBINSize: {err}")
        buf = b" " * size
        err, = nvrtc.nvrtcGetCUBIN(prog, buf)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            raise KernelCompileError(f"nvrtcGetCUBIN: {err}")
        return buf
    finally:
        nvrtc.nvrtcDestroyProgram(prog)


Arg = Union[torch.Tensor, int, float, I64]


class RuntimeKernel:
    """One `extern "C" __global__` function compiled from source at run time."""

    def __init__(self, source: str, function: str, arch: str = "sm_100a", options: Sequence[str] = (),
                 device: Optional[torch.device] = None):
        self.function = function
        self.cubin = compile_cubin(source, f"{function}.cu", arch, options)
        self.device = torch.device(device) if device is not None else None
        self._module = None
        self._func = None

    def _load(self) -> None:
        if self._func is not None:
            return
        from cuda.bindings import driver as drv
        dev = self.device or torch.device("cuda", torch.cuda.current_device())
        torch.cuda.init()
        with torch.cuda.device(dev):
            torch.cuda.current_stream(dev)  # makes PyTorch's primary context current on this thread
            err, mod = drv.cuModuleLoadData(self.cubin)
            if err != drv.CUresult.CUDA_SUCCESS:
                raise RuntimeError(f"cuModuleLoadData: {err}")
            err, fn = drv.cuModuleGetFunction(mod, self.function.encode())
            if err != drv.CUresult.CUDA_SUCCESS:
                raise RuntimeError(f"cuModuleGetFunction({self.function}): {err}")
        self._module, self._func = mod, fn

    @staticmethod
    def _marshal(args: Sequence[Arg]):
        holders = []
        for a in args:
            if isinstance(a, torch.Tensor):
                holders.append(ctypes.c_void_p(a.data_ptr()))
            elif isinstance(a, I64):
                holders.append(ctypes.c_int64(a.value))
            elif isinstance(a, bool) or isinstance(a, int):
                holders.append(ctypes.c_int32(int(a)))
            elif isinstance(a, float):
                holders.append(ctypes.c_float(a))
            else:
                raise TypeError(f"unsupported kernel argument type {type(a).__name__}")
        ptrs = np.array([ctypes.addressof(h) for h in holders], dtype=np.uint64)
        return holders, ptrs

    def launch(self, grid: Tuple[int, int, int], block: Tuple[int, int, int], args: Sequence[Arg],
               shared_bytes: int = 0, stream: Optional[torch.cuda.Stream] = None, sync: bool = False) -> None:
        """Asynchronous launch on `stream` (default: the current stream); `sync` waits for it."""
        from cuda.bindings import driver as drv
        self._load()
        s = stream or torch.cuda.current_stream(self.device)
        holders, ptrs = self._marshal(args)
        err, = drv.cuLaunchKernel(self._func, *grid, *block, shared_bytes, s.cuda_stream, ptrs.ctypes.data, 0)
        if err != drv.CUresult.CUDA_SUCCESS:
            raise RuntimeError(f"cuLaunchKernel({self.function}): {err}")
        if sync:
            s.synchronize()
        del holders

    def launch_1d(self, n: int, args: Sequence[Arg], block: int = 256, stream=None, sync: bool = False) -> None:
        """One thread per element (CudaKernel.Launch1D): grid = ceil(n / block)."""
        self.launch(((n + block - 1) // block, 1, 1), (block, 1, 1), args, 0, stream, sync)

    def close(self) -> None:
        if self._module is not None:
            from cuda.bindings import driver as drv
            drv.cuModuleUnload(self._module)
            self._module = self._func = None
