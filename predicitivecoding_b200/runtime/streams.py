"""Stream pool and events over native streams (C++ in the extension).

Reference: PredictiveCoding.Device/Streams/CudaStreamManager.cs:17-83 (per-thread stream per
device, CreateStream, Synchronize, SynchronizeDevice, RecordEvent, WaitEvent).  Streams come from
a native per-device pool of non-blocking streams at low or high priority and are handed to torch
as external streams, so every kernel of the framework can be issued on them.
"""
from __future__ import annotations

import threading
from typing import Dict

import torch

from .. import ops


class StreamManager:
    _shared = None

    def __init__(self, pool_size: int = 4):
        self.pool_size = pool_size
        self._next: Dict[int, int] = {}
        self._tls = threading.local()

    @classmethod
    def shared(cls) -> "StreamManager":
        if cls._shared is None:
            cls._shared = StreamManager()
        return cls._shared

    def _wrap(self, device: int, handle: int) -> torch.cuda.ExternalStream:
        return torch.cuda.ExternalStream(handle, device=torch.device("cuda", device))

    def create_stream(self, device: int = 0, high_priority: bool = False) -> torch.cuda.ExternalStream:
        i = self._next.get(device, 0)
        self._next[device] = i + 1
        return self._wrap(device, ops.ext().dev_stream(device, i, high_priority, self.pool_size))

    def thread_stream(self, device: int = 0) -> torch.cuda.ExternalStream:
        cache = getattr(self._tls, "streams", None)
        if cache is None:
            cache = self._tls.streams = {}
        if device not in cache:
            cache[device] = self.create_stream(device)
        return cache[device]

    @staticmethod
    def synchronize(stream) -> None:
        stream.synchronize()

    @staticmethod
    def synchronize_device(device: int = 0) -> None:
        torch.cuda.synchronize(device)

    @staticmethod
    def record_event(stream) -> torch.cuda.Event:
        ev = torch.cuda.Event()
        ev.record(stream)
        return ev

    @staticmethod
    def wait_event(event: torch.cuda.Event, stream=None) -> None:
        (stream or torch.cuda.current_stream()).wait_event(event)
