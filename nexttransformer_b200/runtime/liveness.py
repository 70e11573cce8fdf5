"""Host-side rank liveness: a heartbeat in the process group's key-value store.

Every rank records the update it has reached (``beat(step)``) before it launches that update's
work; ``wait_peers(step)`` then waits, with a time limit, until every peer has recorded the same
update.  A rank that died or left between updates never records it, so the others learn of the
failure on the host, before they launch a kernel or a collective that would wait for the missing
rank, and raise ``RankFailure`` naming it.  A rank that leaves on purpose calls ``leave()`` so
the others fail at once instead of at the time limit.

This complements the bounded waits inside the peer-memory kernels (which record an error word
instead of hanging) and the process group's own collective timeout.
"""
import time

import torch.distributed as dist


class RankFailure(RuntimeError):
    """A peer rank stopped taking part in training (died, hung or left)."""

    def __init__(self, ranks, step, reason):
        super().__init__(f"rank(s) {sorted(ranks)} did not reach update {step}: {reason}")
        self.ranks, self.step = sorted(ranks), step


class Heartbeat:
    def __init__(self, store=None, rank=None, world=None, prefix="nt/heartbeat", poll_s=0.05):
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store = store
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.prefix, self.poll_s = prefix, poll_s

    def _key(self, rank):
        return f"{self.prefix}/{rank}"

    def beat(self, step):
        """This rank has reached update ``step``."""
        self.store.set(self._key(self.rank), str(int(step)))

    def leave(self):
        """This rank stops training on purpose (between updates)."""
        self.store.set(self._key(self.rank), "left")

    def _state(self, rank):
        try:
            if not self.store.check([self._key(rank)]):
                return None
            return self.store.get(self._key(rank)).decode()
        except RuntimeError:
            return None

    def wait_peers(self, step, timeout_s=30.0):
        """Wait until every peer has recorded update ``step``; raise ``RankFailure`` otherwise."""
        deadline = time.monotonic() + timeout_s
        waiting = {r for r in range(self.world) if r != self.rank}
        while waiting:
            for r in sorted(waiting):
                state = self._state(r)
                if state == "left":
                    raise RankFailure([r], step, "the rank left training")
                if state is not None and int(state) >= step:
                    waiting.discard(r)
            if not waiting:
                break
            if time.monotonic() > deadline:
                raise RankFailure(waiting, step, f"no heartbeat within {timeout_s:.1f} s")
            time.sleep(self.poll_s)
