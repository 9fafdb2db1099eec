"""Host-side failure detection between ranks.

The reference has no failure detection beyond a barrier around timing and a
per-NEFF runtime watchdog (``contrib/qwen3.6-35b-a3b/BENCHMARK.md:845-851``).
bwn splits the job in two:

* on the device, every spin-wait (peer flags of the fused comm kernels,
  mbarriers) is bounded and reports through the host-mapped status word
  (:func:`bwn.ops.check_status`), so a missing peer never wedges a GPU;
* on the host, :class:`Heartbeat` keeps one key per rank in the rendezvous
  store.  A rank publishes its step before launching it and its error if it
  fails; :meth:`Heartbeat.wait_peers` -- called between steps, with no kernel
  or collective in flight -- raises :class:`PeerFailure` when a peer reported
  an error or stopped advancing, and :class:`ProtocolError` when a peer's
  step counter went backwards or skipped ahead (a corrupted sequence).

Ranks leave only between steps, so the survivors learn of it before their
next launch; a short process-group timeout is the last bound for a rank that
dies inside a collective.
"""
from __future__ import annotations

import json
import time


class PeerFailure(RuntimeError):
    pass


class ProtocolError(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store, rank: int, world: int, prefix: str = "bwn/hb", stale_s: float = 5.0):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.stale_s = prefix, stale_s
        self._last: dict[int, tuple[int, float]] = {}

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def _err_key(self, r: int) -> str:
        return f"{self.prefix}/err/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank), json.dumps({"step": int(step)}))

    def report_error(self, msg: str) -> None:
        self.store.set(self._err_key(self.rank), str(msg)[:2000])

    def _peek(self, key: str):
        return self.store.get(key).decode() if self.store.check([key]) else None

    def poll(self, step: int) -> dict[int, int]:
        """One non-blocking look at every peer; raises on reported errors or
        broken sequences, returns ``{rank: step}`` of the peers seen."""
        now = time.monotonic()
        seen = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            err = self._peek(self._err_key(r))
            if err is not None:
                raise PeerFailure(f"rank {r} reported an error: {err}")
            raw = self._peek(self._key(r))
            if raw is None:
                continue
            s = int(json.loads(raw)["step"])
            prev = self._last.get(r)
            if prev is not None and s < prev[0]:
                raise ProtocolError(f"rank {r} step went backwards ({prev[0]} -> {s})")
            if s > step + 1:
                raise ProtocolError(f"rank {r} is at step {s} while this rank waits for step {step}")
            if prev is None or s != prev[0]:
                self._last[r] = (s, now)
            seen[r] = s
        return seen

    def wait_peers(self, step: int, timeout_s: float | None = None, interval_s: float = 0.01) -> None:
        """Block until every peer has published ``step`` (or later); raise when a
        peer failed, broke the sequence, or made no progress for ``stale_s``."""
        t0 = time.monotonic()
        limit = self.stale_s if timeout_s is None else timeout_s
        while True:
            seen = self.poll(step)
            behind = [r for r in range(self.world) if r != self.rank and seen.get(r, -1) < step]
            if not behind:
                return
            now = time.monotonic()
            stale = [r for r in behind if now - self._last.get(r, (None, t0))[1] > self.stale_s]
            if stale or now - t0 > limit:
                raise PeerFailure(f"ranks {stale or behind} made no progress to step {step} "
                                  f"within {self.stale_s if stale else limit:.1f}s (dead or hung)")
            time.sleep(interval_s)


def guarded(hb: Heartbeat, step: int, fn, *args, **kwargs):
    """Run one step: publish it, run ``fn``; on an exception publish the error
    (so peers stop before their next launch) and re-raise."""
    hb.beat(step)
    try:
        return fn(*args, **kwargs)
    except BaseException as e:
        hb.report_error(f"step {step}: {type(e).__name__}: {e}")
        raise
