"""Host-side liveness of tensor-parallel ranks.

A tensor-parallel generation (InferenceAPI.init_tensor_parallel) runs NCCL all-reduces inside
every target forward; a rank that dies leaves the others' next collective waiting for it.
PeerMonitor lets the ranks learn of a lost peer on the host, between steps, before any rank
launches the next step's collectives: each rank announces the step it is about to run in a
shared key-value store (the torch.distributed store the ranks already use to exchange the
NCCL id, or any object with set / get / check), and waits, with a bound, until every peer has
announced the same step.  A peer that has left (its process ended, or it raised and called
leave()) or that does not show up within the timeout raises PeerLost on every surviving rank.

This is the first line of defence; the library's ulb_tp_set_timeout (InferenceAPI.
set_collective_timeout) is the second, for a peer lost while a collective is in flight: the
survivor's wait is bounded and the communicator aborted.  The reference has no multi-GPU data
path (src/vulkan_backend/multi_gpu_manager.cpp enumerates devices and splits host arrays).
"""
import time


class PeerLost(RuntimeError):
    """A tensor-parallel peer left or stopped answering; `ranks` lists the missing ones."""

    def __init__(self, ranks, step, why):
        super().__init__("tensor-parallel rank(s) %s %s before step %d" % (sorted(ranks), why, step))
        self.ranks = sorted(ranks)
        self.step = step


class PeerMonitor:
    """store: set(key, bytes|str), get(key) -> bytes, check([key]) -> bool (a torch.distributed
    Store).  timeout_s bounds each wait_step."""

    def __init__(self, store, rank, world, timeout_s=30.0, prefix="ulb/tp", poll_s=0.02):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix, self.poll_s = float(timeout_s), prefix, poll_s

    def _key(self, what, rank):
        return "%s/%s/%d" % (self.prefix, what, rank)

    def leave(self):
        """Announce that this rank is leaving (call from a finally block or an exception handler)."""
        self.store.set(self._key("left", self.rank), "1")

    def wait_step(self, step):
        """Announce `step` and return once every peer has announced it (or a later one); raise
        PeerLost if a peer left or did not arrive within the timeout."""
        self.store.set(self._key("step", self.rank), str(step))
        deadline = time.monotonic() + self.timeout_s
        pending = set(r for r in range(self.world) if r != self.rank)
        while pending:
            for r in list(pending):
                k = self._key("step", r)
                if self.store.check([k]) and int(self.store.get(k)) >= step:
                    pending.discard(r)  # it reached this step (whatever it did after)
                elif self.store.check([self._key("left", r)]):
                    raise PeerLost([r], step, "left")
            if not pending:
                break
            if time.monotonic() >= deadline:
                raise PeerLost(pending, step, "did not arrive within %.1f s" % self.timeout_s)
            time.sleep(self.poll_s)
