"""Failure detection for multi-rank jobs: heartbeats through the rendezvous store, a step watchdog,
and a check of the device error word written by the bounded in-kernel waits.

The reference has no health checks (graceful cancellation, NaN guards and recover-on-open are its
only defences; PredictiveCoding.Device/Training/DevicePretrainer.cs:141-149,205-219,
PredictiveCoding.LLM/Training/Optimizers.cs:100-104).  Here:

* ``Heartbeat`` -- every rank's background thread stamps ``hb/<rank>`` in the torch.distributed
  store; ``dead_ranks()`` lists ranks whose stamp is older than the timeout (a rank that crashed,
  exited or never joined).  Ranks call ``check()`` between steps, before launching work that
  contains collectives, so a survivor raises ``PeerFailure`` on the host instead of entering a
  collective that can never complete.
* ``Watchdog`` -- a thread that fires a callback when ``kick()`` has not been called for
  ``timeout`` seconds (a step that hangs on the host or never returns from the device).
* ``check_device_error(err)`` -- raises when a peer-memory kernel recorded a timed-out wait (the
  kernels never trap: they record the code and return, leaving the context usable).
"""
from __future__ import annotations

import threading
import time
from typing import Callable, List, Optional

import torch


class PeerFailure(RuntimeError):
    def __init__(self, ranks: List[int], what: str = "heartbeat"):
        super().__init__(f"ranks {ranks} stopped responding ({what})")
        self.ranks = ranks


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.2, timeout: float = 2.0,
                 prefix: str = "hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.started = time.time()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), repr(time.time()))

    def start(self) -> "Heartbeat":
        self.beat()

        def run():
            while not self._stop.wait(self.interval):
                try:
                    self.beat()
                except Exception:
                    return

        self._thread = threading.Thread(target=run, daemon=True, name=f"heartbeat-{self.rank}")
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval + 1)

    def last_seen(self, r: int) -> Optional[float]:
        try:
            if not self.store.check([self._key(r)]):
                return None
            return float(self.store.get(self._key(r)).decode())
        except Exception:
            return None

    def dead_ranks(self) -> List[int]:
        now = time.time()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            t = self.last_seen(r)
            if t is None:
                if now - self.started > self.timeout:   # never joined
                    dead.append(r)
            elif now - t > self.timeout:
                dead.append(r)
        return dead

    def check(self) -> None:
        dead = self.dead_ranks()
        if dead:
            raise PeerFailure(dead)

    def attribute(self) -> List[int]:
        """After a collective failed: wait one timeout and name the ranks whose heartbeat stopped."""
        time.sleep(self.timeout + 2 * self.interval)
        return self.dead_ranks()

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()


class Watchdog:
    def __init__(self, timeout: float, on_timeout: Callable[[float], None], poll: float = 0.05):
        self.timeout, self.on_timeout, self.poll = timeout, on_timeout, poll
        self._last = time.monotonic()
        self._stop = threading.Event()
        self.fired = False
        self._thread = threading.Thread(target=self._run, daemon=True, name="watchdog")

    def kick(self) -> None:
        self._last = time.monotonic()

    def _run(self) -> None:
        while not self._stop.wait(self.poll):
            idle = time.monotonic() - self._last
            if idle > self.timeout and not self.fired:
                self.fired = True
                self.on_timeout(idle)

    def start(self) -> "Watchdog":
        self.kick()
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(timeout=1.0)

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()


def check_device_error(err: torch.Tensor, what: str = "peer kernel") -> None:
    """Raise if a bounded device wait recorded a timeout (err is the kernels' int32 error word)."""
    code = int(err.item())
    if code:
        names = {1: "TMA stage never filled", 2: "stage never released", 3: "accumulator never ready",
                 4: "accumulator never drained", 5: "peer flag never arrived", 7: "gathered chunk never copied"}
        raise PeerFailure([], f"{what}: device error {code} ({names.get(code, 'unknown')})")
