"""Failure detection between ranks: heartbeats on the c10d store, and host-side fault
injection for tests.

The reference has no failure detection (no timeouts configured, no heartbeat; a dead
rank leaves the others blocked in their next NCCL call).  Here:

* :class:`Heartbeat` — a daemon thread per rank bumps ``hb/<rank>`` (a counter) on
  the process group's TCPStore every ``interval`` seconds and watches every peer's
  counter.  A peer whose counter has not moved for ``timeout`` seconds (measured on
  this rank's clock, so hosts need no clock sync), or that published ``hb/<rank>/exit``
  with a non-zero code, is reported dead.  ``check()`` raises :class:`PeerFailure` on
  the host; the trainer calls it between steps, before launching the next step's
  kernels and collectives, so no rank ever enters a collective its peer left.
* device-side waits are bounded separately (``TT_COMM_TIMEOUT_S`` in the comm runtime;
  the process group's own timeout for NCCL), so a rank that dies inside a step ends
  the others' next collective with an error instead of a hang.
* :func:`fault_point` — host-side fault injection driven by ``TT_FAULT_INJECT``
  (comma-separated ``kind@rank[:step]``):

  - ``exit@R:S``          rank R raises :class:`InjectedFault` at the start of step S
                          (between steps: no kernel or collective of its in flight);
  - ``hang_heartbeat@R``  rank R's heartbeat thread stops publishing (a silent rank);
  - ``skip_signal@R``     rank R skips the signal of its next symmetric-heap barrier,
                          so its peers' bounded device waits expire and report a status
                          code (see ``tinytron_b200.parallel.symm``).

Nothing here faults, traps or hangs a GPU: injected failures happen on the host.
"""
from __future__ import annotations

import os
import threading
import time


class PeerFailure(RuntimeError):
    """A peer rank stopped heartbeating or exited with an error."""

    def __init__(self, ranks, reason: str):
        super().__init__(f"peer rank(s) {sorted(ranks)} failed: {reason}")
        self.ranks = sorted(ranks)
        self.reason = reason


class InjectedFault(RuntimeError):
    """Raised by :func:`fault_point` for an injected failure."""


# ---------------------------------------------------------------------------- fault injection
def parse_fault_spec(spec: str | None = None) -> list[tuple[str, int, int | None]]:
    spec = os.environ.get("TT_FAULT_INJECT", "") if spec is None else spec
    out = []
    for item in filter(None, (s.strip() for s in spec.split(","))):
        kind, _, where = item.partition("@")
        rank_s, _, step_s = where.partition(":")
        if not kind or not rank_s:
            raise ValueError(f"bad TT_FAULT_INJECT entry {item!r}; expected kind@rank[:step]")
        out.append((kind, int(rank_s), int(step_s) if step_s else None))
    return out


def fault_active(kind: str, rank: int, step: int | None = None, spec: str | None = None) -> bool:
    for k, r, s in parse_fault_spec(spec):
        if k == kind and r == rank and (s is None or step is None or s == step):
            return True
    return False


def fault_point(kind: str, rank: int, step: int | None = None) -> None:
    """Raise :class:`InjectedFault` when ``kind@rank[:step]`` is injected."""
    if fault_active(kind, rank, step):
        raise InjectedFault(f"injected fault {kind} on rank {rank}" + (f" at step {step}" if step is not None else ""))


# ---------------------------------------------------------------------------- heartbeat
def default_store():
    """The default process group's c10d store (TCPStore under env:// rendezvous)."""
    import torch.distributed as dist
    from torch.distributed import distributed_c10d as c10d

    if not dist.is_initialized():
        raise RuntimeError("Heartbeat needs an initialised process group (or an explicit store)")
    return c10d._get_default_store()


class Heartbeat:
    def __init__(self, rank: int, world: int, store=None, interval: float = 1.0, timeout: float = 30.0,
                 prefix: str = "tt_hb", start: bool = True):
        self.rank, self.world = rank, world
        self.store = store if store is not None else default_store()
        self.interval, self.timeout = float(interval), float(timeout)
        self.prefix = prefix
        self._seq = 0
        self._last = {r: (-1, time.monotonic()) for r in range(world) if r != rank}
        self._dead: dict[int, str] = {}
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self._silent = fault_active("hang_heartbeat", rank)
        self._thread = threading.Thread(target=self._run, name=f"tt-heartbeat-{rank}", daemon=True)
        self._beat()
        if start:
            self._thread.start()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _beat(self) -> None:
        if self._silent:
            return
        self._seq += 1
        self.store.set(self._key(self.rank), str(self._seq))

    def poll(self) -> None:
        """One round: publish our counter, read every peer's (also called by the thread)."""
        self._beat()
        now = time.monotonic()
        for r in list(self._last):
            if r in self._dead:
                continue
            exit_key = f"{self._key(r)}/exit"
            if self.store.check([exit_key]):
                code = int(self.store.get(exit_key).decode() or "0")
                if code != 0:
                    self._mark(r, f"exited with code {code}")
                else:
                    self._last.pop(r, None)  # clean exit: stop watching
                continue
            seq = int(self.store.get(self._key(r)).decode()) if self.store.check([self._key(r)]) else -1
            last_seq, since = self._last[r]
            if seq != last_seq:
                self._last[r] = (seq, now)
            elif now - since > self.timeout:
                self._mark(r, f"no heartbeat for {now - since:.1f} s")

    def _mark(self, r: int, why: str) -> None:
        with self._lock:
            self._dead.setdefault(r, why)

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.poll()
            except Exception as exc:  # the store itself is gone: the master rank died
                self._mark(-1, f"store unreachable: {exc}")

    def dead(self) -> dict[int, str]:
        with self._lock:
            return dict(self._dead)

    def check(self) -> None:
        d = self.dead()
        if d:
            raise PeerFailure(d.keys(), "; ".join(f"rank {r}: {w}" for r, w in sorted(d.items())))

    def close(self, exit_code: int = 0) -> None:
        """Stop the thread and publish this rank's exit code (0: clean)."""
        self._stop.set()
        if self._thread.is_alive():
            self._thread.join(timeout=5)
        try:
            self.store.set(f"{self._key(self.rank)}/exit", str(int(exit_code)))
        except Exception:
            pass
