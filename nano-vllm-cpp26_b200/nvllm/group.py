"""Failure detection between the steps of a multi-GPU group (one process per GPU).

The reference is one CPU process; here the head split and the head-parallel
model run one process per GPU whose kernels wait on each other's flags, and
the benchmarks take collectives between steps. A rank that raises, exits or
never arrives must not leave the others waiting. Three layers:

* :class:`StepGuard` (host, between steps): before launching step i every rank
  announces i in the group's key-value store and waits, with a limit, until
  every peer has announced i too. A peer that announced it left
  (:meth:`StepGuard.leave`, or :meth:`StepGuard.fail` from an exception
  handler) or stays silent past the limit makes :meth:`StepGuard.enter` raise
  :class:`PeerLost` before this rank launches anything that would wait for it.
* the device waits themselves are bounded (2 s, then NVLLM_ERR_TIMEOUT in
  nvllm_get_last_error), so a peer lost inside a step cannot hang a GPU;
* :func:`abort_group` ends the process group without a rendezvous (with NCCL,
  ncclCommAbort on its communicators), so no collective already queued on this
  rank waits for the lost peer either. Process groups are created with a short
  timeout (:func:`init_group`) as the last bound.

Nothing here touches a GPU: the tests run it as gloo ranks on the CPU.
"""
from __future__ import annotations

import datetime
import time


class PeerLost(RuntimeError):
    """A peer left or stopped answering between steps."""

    def __init__(self, ranks, step: int, why: str):
        self.ranks = sorted(ranks)
        self.step = step
        self.why = why
        super().__init__(f"rank(s) {self.ranks} {why} before step {step}")


class StepGuard:
    """Step admission over a torch.distributed store (TCPStore, FileStore...).

    ``timeout_s`` bounds how long :meth:`enter` waits for a silent peer; keys
    live under ``prefix`` so that several groups can share one store."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0,
                 poll_s: float = 0.002, prefix: str = "nvllm/guard"):
        self.store = store
        self.rank, self.world = rank, world
        self.timeout_s, self.poll_s = timeout_s, poll_s
        self.prefix = prefix
        self.peers = [r for r in range(world) if r != rank]

    def _key(self, kind: str, rank: int) -> str:
        return f"{self.prefix}/{kind}/{rank}"

    def enter(self, step: int) -> None:
        """Announces ``step`` and returns once every peer has announced it (or
        a later one); raises :class:`PeerLost` if one left or stays silent
        for ``timeout_s``."""
        self.store.set(self._key("step", self.rank), str(step))
        waiting = set(self.peers)
        deadline = time.monotonic() + self.timeout_s
        while waiting:
            for r in sorted(waiting):
                if self.store.check([self._key("left", r)]):
                    why = self.store.get(self._key("left", r)).decode()
                    raise PeerLost([r], step, f"left ({why})")
                k = self._key("step", r)
                if self.store.check([k]) and int(self.store.get(k)) >= step:
                    waiting.discard(r)
            if not waiting:
                return
            if time.monotonic() > deadline:
                raise PeerLost(waiting, step, f"silent for {self.timeout_s:.1f} s")
            time.sleep(self.poll_s)

    def leave(self, why: str = "done") -> None:
        """Tells the peers, between steps, that this rank takes no further step."""
        self.store.set(self._key("left", self.rank), why)

    def fail(self, exc: BaseException) -> None:
        """:meth:`leave` from an exception handler, naming the exception."""
        self.leave(f"error: {type(exc).__name__}: {exc}"[:200])


def init_group(backend: str, rank: int, world: int, master: str, timeout_s: float = 30.0,
               **kw):
    """``torch.distributed.init_process_group`` with a short timeout (the last
    bound on a collective whose peer is gone) over ``tcp://master``."""
    import torch.distributed as dist
    dist.init_process_group(backend, init_method=f"tcp://{master}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist


def abort_group() -> None:
    """Ends the default process group without waiting for its peers (NCCL:
    ncclCommAbort on its communicators); a later collective on it fails at once
    instead of waiting."""
    import torch.distributed as dist
    if not dist.is_initialized():
        return
    try:
        from torch.distributed.distributed_c10d import _abort_process_group
        _abort_process_group()
    except Exception:  # older torch, or a backend without abort: plain teardown
        dist.destroy_process_group()
