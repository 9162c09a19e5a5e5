"""Host-side failure detection for the ranks of a group: heartbeats and failure notices in the process
group's key-value store, checked between steps, before the next launch.

The reference has none: its product kernel spins without bound (exp/M17_epoch_ab/fused_ar_norm_nf.cu:95-96,
181-183), launches run under a wall-clock `timeout` (exp/M17_epoch_ab/run.py:52), and a mismatched warm-up
was only caught by NCCL's watchdog (exp/M18_incremental/README.md:52). Here every device wait is already
bounded (the kernels set an error word that `TPCommunicator.check()` turns into `TPCommTimeout`); this
module covers what a kernel cannot see: a rank that raised, exited, left or never joined. Such a rank
must not leave its peers inside a collective or a peer-memory wait, so each rank

  * beats (`beat()`): increments its counter key - no clocks are compared across processes; a peer is
    stale when its counter has not moved for `stale_s` seconds of the observer's own clock;
  * posts a notice when it fails (`fail(reason)`, or `guard()` around a step) or leaves (`leave()`);
  * checks its peers (`check()`) between steps and raises `RankFailure` naming the ranks and why,
    before it launches anything that needs them.

`wait_joined(timeout_s)` at start-up turns a rank that never arrives into the same error.

    mon = RankMonitor.from_default_group(stale_s=30)
    mon.wait_joined(60)
    for step in range(n):
        mon.sync(30)                 # every peer reached this step, or RankFailure (failed / left / late)
        with mon.guard():            # an exception here is posted for the peers, then re-raised
            runner.step(batch)

`check()` is the cheaper non-blocking form (notices and stale heartbeats only) for loops that beat on
their own.
"""
from __future__ import annotations

import contextlib
import time


class RankFailure(RuntimeError):
    """Peers that failed, left or stopped beating: {rank: reason}."""

    def __init__(self, problems: dict[int, str]):
        self.problems = dict(problems)
        super().__init__("; ".join(f"rank {r}: {why}" for r, why in sorted(self.problems.items())))


class RankMonitor:
    def __init__(self, store, rank: int, world: int, prefix: str = "cob/health", stale_s: float = 30.0,
                 clock=time.monotonic):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.stale_s, self.clock = prefix, stale_s, clock
        self._seen: dict[int, tuple[int, float]] = {}  # peer -> (last counter value, when it last moved)
        self.beats = 0

    @classmethod
    def from_default_group(cls, **kw) -> "RankMonitor":
        import torch.distributed as dist

        store = dist.distributed_c10d._get_default_store()
        return cls(store, dist.get_rank(), dist.get_world_size(), **kw)

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def _has(self, key: str) -> bool:
        return bool(self.store.check([key]))  # non-blocking existence test

    # ---- this rank
    def beat(self):
        self.beats = int(self.store.add(self._key("hb", self.rank), 1))

    def fail(self, reason: str):
        self.store.set(self._key("fail", self.rank), reason[:500])

    def leave(self):
        self.store.set(self._key("left", self.rank), "1")

    @contextlib.contextmanager
    def guard(self):
        """Post any exception of the block as this rank's failure, then re-raise it."""
        try:
            yield self
        except BaseException as e:
            try:
                self.fail(f"{type(e).__name__}: {e}")
            finally:
                raise

    # ---- peers
    def problems(self) -> dict[int, str]:
        now = self.clock()
        out = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            if self._has(self._key("fail", r)):
                out[r] = "failed: " + self.store.get(self._key("fail", r)).decode(errors="replace")
                continue
            if self._has(self._key("left", r)):
                out[r] = "left the group"
                continue
            n = int(self.store.add(self._key("hb", r), 0))  # read without changing it
            last = self._seen.get(r)
            if last is None or n != last[0]:
                self._seen[r] = (n, now)
            elif now - last[1] > self.stale_s:
                out[r] = f"no heartbeat for {now - last[1]:.1f} s (counter stuck at {n})"
        return out

    def check(self):
        p = self.problems()
        if p:
            raise RankFailure(p)

    def sync(self, timeout_s: float, poll_s: float = 0.001):
        """Step boundary: beat, then wait until every peer has beaten as often as this rank (it reached the
        same step) or raise RankFailure for peers that failed, left, or did not arrive within timeout_s.
        Host-only; a rank that leaves between steps posts `leave()` instead of beating."""
        self.beat()
        target, t0 = self.beats, self.clock()
        while True:
            behind = {r for r in range(self.world)
                      if r != self.rank and int(self.store.add(self._key("hb", r), 0)) < target}
            if not behind:
                return
            # a notice read after the counter: re-read the counter, since a peer beats before it posts a
            # notice (one store, so the order holds) - it may have reached this step and left afterwards
            failed = {r: why for r, why in self.problems().items()
                      if r in behind and int(self.store.add(self._key("hb", r), 0)) < target}
            if failed:
                raise RankFailure(failed)
            if self.clock() - t0 > timeout_s:
                raise RankFailure({r: f"did not reach step {target} within {timeout_s:.1f} s" for r in behind})
            time.sleep(poll_s)

    def wait_joined(self, timeout_s: float, poll_s: float = 0.05):
        """Beat once, then wait until every peer has beaten at least once (or raise RankFailure)."""
        self.beat()
        t0 = self.clock()
        while True:
            missing = {r for r in range(self.world)
                       if r != self.rank and int(self.store.add(self._key("hb", r), 0)) == 0}
            failed = self.problems()
            if failed:
                raise RankFailure(failed)
            if not missing:
                return
            if self.clock() - t0 > timeout_s:
                raise RankFailure({r: f"never joined within {timeout_s:.1f} s" for r in missing})
            time.sleep(poll_s)
