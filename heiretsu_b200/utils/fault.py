"""Host-side failure detection: per-rank heartbeats and a watchdog thread.

The reference has no failure handling at all: a rank that dies or stalls
leaves its peers blocked in the next collective until NCCL's default
timeout (train.py:250-258 sets none). Here every rank

  * publishes ``(step, state)`` under ``<prefix>/beat/<rank>`` in the
    torch.distributed key-value store after each completed step,
  * publishes ``<prefix>/failed`` (rank and reason) when it leaves through
    an exception, so peers learn of it without waiting for a timeout,
  * runs a watchdog thread that polls the store and records a failure when
    a peer announced one, or when a peer's beat has not changed for
    ``timeout_s`` seconds of this rank's clock (no cross-host clock needed).

The training loop calls :meth:`StepWatchdog.check` between steps, before it
launches any kernel or collective of the next step, and gets a
:class:`PeerFailure` instead of entering a collective that can never
complete. Only host state is involved: nothing here waits on, or touches,
a GPU.
"""
from __future__ import annotations

import threading
import time
from typing import Dict, Optional, Tuple


class PeerFailure(RuntimeError):
    """A peer rank failed (announced) or stopped making progress (timed out)."""

    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank}: {reason}")
        self.rank = rank
        self.reason = reason


def default_store():
    """The store of the default process group (the torchrun rendezvous store)."""
    import torch.distributed as dist
    from torch.distributed import distributed_c10d as c10d

    if not dist.is_initialized():
        raise RuntimeError("default_store: torch.distributed is not initialised")
    return c10d._get_default_store()


class StepWatchdog:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 300.0, poll_s: float = 0.25,
                 prefix: str = "hb_watchdog", start: bool = True):
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = float(timeout_s)
        self.poll_s = float(poll_s)
        self.prefix = prefix
        self._failure: Optional[Tuple[int, str]] = None
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._seen: Dict[int, Tuple[str, float]] = {}
        self._thread: Optional[threading.Thread] = None
        self.beat(0, "start")
        if start:
            self.start()

    # -- this rank ------------------------------------------------------------
    def _key(self, what: str) -> str:
        return f"{self.prefix}/{what}"

    def beat(self, step: int, state: str = "run") -> None:
        self.store.set(self._key(f"beat/{self.rank}"), f"{step}:{state}")

    def mark_failed(self, reason: str) -> None:
        """Announce that this rank is leaving because of an error."""
        try:
            self.store.set(self._key("failed"), f"{self.rank}:{reason[:200]}")
        except Exception:
            pass  # the store itself may be gone; peers then time out instead

    def finish(self) -> None:
        """Normal exit: peers must not read the silence that follows as a stall."""
        self.beat(-1, "done")
        self.stop()

    # -- peers ----------------------------------------------------------------
    def _poll_once(self) -> None:
        now = time.monotonic()
        if self.store.check([self._key("failed")]):
            raw = self.store.get(self._key("failed")).decode()
            r, _, why = raw.partition(":")
            if int(r) != self.rank:
                self._set_failure(int(r), f"announced failure: {why}")
                return
        for r in range(self.world):
            if r == self.rank:
                continue
            key = self._key(f"beat/{r}")
            val = self.store.get(key).decode() if self.store.check([key]) else "absent"
            if val.endswith(":done"):
                self._seen[r] = (val, now)
                continue
            prev = self._seen.get(r)
            if prev is None or prev[0] != val:
                self._seen[r] = (val, now)
            elif now - prev[1] > self.timeout_s:
                self._set_failure(r, f"no progress for {now - prev[1]:.1f}s (last beat {val})")
                return

    def _set_failure(self, rank: int, reason: str) -> None:
        with self._lock:
            if self._failure is None:
                self._failure = (rank, reason)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self._poll_once()
            except Exception as e:  # store unreachable: the rendezvous host is gone
                self._set_failure(-1, f"store unreachable: {type(e).__name__}")
            if self._failure is not None:
                return
            self._stop.wait(self.poll_s)

    def start(self) -> None:
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="hb-watchdog", daemon=True)
            self._thread.start()

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5 * self.poll_s + 1)
            self._thread = None

    @property
    def failure(self) -> Optional[Tuple[int, str]]:
        with self._lock:
            return self._failure

    def check(self) -> None:
        """Raise PeerFailure if a peer failed; call between steps."""
        f = self.failure
        if f is not None:
            raise PeerFailure(*f)
