"""The multi-rank host logic on the CPU (gloo, world size 2): sequence
partitioning gives each rank its own batch of the same total size (the same
context lengths in another order, other blocks), the timing reduction takes the
maximum over ranks, and the handle exchange of the head split gives every rank
every peer's handles in rank order."""
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import sys
    from pathlib import Path

    import torch
    import torch.distributed as dist
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "nano-vllm-cpp26_b200"))
    from nvllm.workload import make_batch
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60))
        spec = make_batch("decode", seed=0, rank=rank)  # as bench.py builds rank r's batch
        mine = (rank, spec.ctx_lens.tolist(), bytes([rank]) * 64, spec.block_tables[:, 0].tolist(),
                spec.decode_algorithmic_bytes())
        every = [None] * world
        dist.all_gather_object(every, mine)
        t = torch.tensor([0.5 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, every, float(t.item()), None))
    except Exception as exc:  # reported to the parent
        q.put((rank, None, None, repr(exc)))


def test_two_rank_host_logic():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    results.sort()
    for rank, every, tmax, err in results:
        assert err is None, err
        assert [e[0] for e in every] == list(range(world))  # rank order
        assert every[rank][2] == bytes([rank]) * 64
        assert tmax == pytest.approx(0.5 + world - 1)
    every = results[0][1]
    ctxs = [np.array(e[1]) for e in every]
    assert not np.array_equal(ctxs[0], ctxs[1])  # each rank serves its own sequences
    assert np.array_equal(np.sort(ctxs[0]), np.sort(ctxs[1]))  # of the same lengths
    assert every[0][3] != every[1][3]  # in other physical blocks
    assert every[0][4] == every[1][4]  # so every GPU moves the same bytes
    assert all(((c >= 512) & (c <= 4096)).all() and len(c) == 64 for c in ctxs)
