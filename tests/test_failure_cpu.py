"""Failure detection between steps on the CPU (gloo ranks, no GPU).

A rank of a multi-GPU group that exits, raises or never arrives between steps
must not leave the others waiting: the survivors' StepGuard.enter raises
PeerLost before their next launch (at once when the peer said it left, within
the guard's limit when it went silent), and a collective taken anyway ends with
an error within the process group's short timeout instead of waiting.
"""
import datetime
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, ports, mode, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nano-vllm-cpp26_b200"))
    import torch
    import torch.distributed as dist

    from nvllm.group import PeerLost, StepGuard, abort_group, init_group
    init_group("gloo", rank, world, f"127.0.0.1:{ports[0]}", timeout_s=3.0)
    store = dist.TCPStore("127.0.0.1", ports[1], world, rank == 0,
                          timeout=datetime.timedelta(seconds=30))
    guard = StepGuard(store, rank, world, timeout_s=1.5)
    doomed = rank == world - 1
    t = torch.ones(1)
    events = []
    try:
        for step in range(4):
            if doomed and step == 1:
                if mode == "raise":
                    try:
                        raise ValueError("a bad batch")
                    except ValueError as exc:
                        guard.fail(exc)
                        q.put((rank, ["raised"], None))
                        return
                if mode == "exit":
                    q.put((rank, ["exited"], None))
                    q.close()
                    q.join_thread()  # the parent gets the note; the peers get nothing
                    os._exit(0)  # gone without a word, between steps
                if mode == "leave":
                    guard.leave()
                    q.put((rank, ["left"], None))
                    return
            guard.enter(step)
            dist.all_reduce(t)  # the step's collective
            events.append(("step", step))
    except PeerLost as exc:
        t0 = time.monotonic()
        events.append(("lost", exc.ranks, exc.step, exc.why.split(" ")[0]))
        if mode == "exit":
            # a collective taken anyway ends within the group's timeout
            try:
                dist.all_reduce(t)
                events.append(("collective", "returned"))
            except Exception:
                events.append(("collective", "error", time.monotonic() - t0 < 20.0))
        abort_group()
        q.put((rank, events, None))
        return
    except Exception as exc:  # reported to the parent
        q.put((rank, events, repr(exc)))
        return
    q.put((rank, events, "no PeerLost"))


@pytest.mark.parametrize("mode", ["raise", "leave", "exit"])
def test_survivors_learn_of_a_lost_rank_between_steps(mode):
    world = 3
    ports = (_free_port(), _free_port())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, ports, mode, q)) for r in range(world)]
    t0 = time.monotonic()
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, events, err = q.get(timeout=120)
        results[rank] = (events, err)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode is not None, "a rank is still waiting"
    assert time.monotonic() - t0 < 90
    for rank in range(world - 1):
        events, err = results[rank]
        assert err is None, err
        assert events[0] == ("step", 0)
        lost = [e for e in events if e[0] == "lost"]
        assert lost, events
        _, ranks, step, why = lost[0]
        assert ranks == [world - 1] and step == 1, lost
        assert why == ("silent" if mode == "exit" else "left"), lost
        if mode == "exit":
            assert ("collective", "error", True) in events, events
