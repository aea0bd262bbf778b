"""Tracing and timing: NVTX ranges per phase, torch.profiler traces, device step timing.

The reference has no profiler integration (its observability is Stopwatch medians, tokens/s in the
pretraining progress record and the activation probe).  Here:

* ``nvtx_range(name)`` marks a phase for Nsight tools; ranges are emitted only when tracing is on
  (``PCB_NVTX=1`` or ``set_tracing(True)``), so the hot loop pays nothing by default.  Ranges
  recorded while a CUDA graph is captured are host-side only and cost nothing at replay;
* ``profile_steps`` runs a step function under ``torch.profiler`` and writes a Chrome trace;
* ``DeviceTimer`` brackets work with CUDA events on the launching stream and, with a process group,
  reports the maximum over ranks (how every multi-GPU number in this package is quoted).
"""
from __future__ import annotations

import contextlib
import os
from typing import Callable, Optional

import torch

_TRACING = os.environ.get("PCB_NVTX", "0") == "1"


def set_tracing(on: bool) -> None:
    global _TRACING
    _TRACING = bool(on)


def tracing() -> bool:
    return _TRACING


@contextlib.contextmanager
def nvtx_range(name: str):
    if _TRACING and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def profile_steps(step: Callable[[], None], steps: int, path: str, warmup: int = 1) -> str:
    """Run `warmup` untraced then `steps` traced calls of `step`; write a Chrome trace to `path`."""
    for _ in range(warmup):
        step()
    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)
        torch.cuda.synchronize()
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(steps):
            step()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    prof.export_chrome_trace(path)
    return path


class DeviceTimer:
    """CUDA-event timing on the current stream; `elapsed_ms()` is the max over `group`'s ranks."""

    def __init__(self, device: Optional[torch.device] = None, group=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.group = group
        self.start = torch.cuda.Event(enable_timing=True)
        self.end = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        torch.cuda.synchronize(self.device)
        self.start.record(torch.cuda.current_stream(self.device))
        return self

    def __exit__(self, *exc):
        self.end.record(torch.cuda.current_stream(self.device))
        torch.cuda.synchronize(self.device)
        return False

    def elapsed_ms(self) -> float:
        ms = self.start.elapsed_time(self.end)
        import torch.distributed as dist
        if self.group is not None and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            t = torch.tensor([ms], device=self.device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            ms = float(t)
        return ms
