"""The continuous-batching scheduler (nvllm_scheduler_*, host library) against
the reference's own scheduler: fed the reference's requests and, after each
step, the tokens the reference sampled, it must produce the same batch as the
reference at every step — the same sequences in the same order, the same
computed / total lengths and uncomputed tokens, and bit-identical block tables
(src/scheduler.cpp:30-121, :123-198 with src/kv_cache.cpp's FIFO allocator)."""
import numpy as np
import pytest

from helpers import load_trace, trace_requests

TRACES = ("tokens_toy_seeded", "tokens_toy_bench", "tokens_wide")


@pytest.mark.parametrize("name", TRACES)
def test_scheduler_replays_reference_batches(name):
    from nvllm.host import BlockAllocator, Scheduler
    cfg, z, steps = load_trace(name)
    max_batch, max_tokens, watermark = (int(x) for x in z["sched"])
    blocks = BlockAllocator(int(z["num_blocks"]))
    sched = Scheduler(int(z["block_size"]), max_batch, max_tokens, watermark)
    prompts, max_new = trace_requests(z)
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        sched.add_request(i + 1, p, m)
    for i, st in enumerate(steps):
        summary = sched.schedule_step(blocks)
        assert summary["batch_size"] == len(st["seqs"])
        assert np.array_equal(sched.batch_record(i), st["record"]), f"{name} step {i}"
        sched.process_outputs(blocks, st["sampled"])
    c = sched.counts()
    assert c["running"] == 0 and c["waiting"] == 0 and c["completed"] == len(prompts)
    assert blocks.num_free() == int(z["num_blocks"])


def test_seeded_trace_exercises_preemption():
    """The tight arena of tokens_toy_seeded preempts: sequences come back with
    no computed tokens after having run, and the replay counts them."""
    from nvllm.host import BlockAllocator, Scheduler
    cfg, z, steps = load_trace("tokens_toy_seeded")
    seen, recomputed = set(), 0
    for st in steps:
        for s in st["seqs"]:
            if s["seq_id"] in seen and s["num_computed"] == 0:
                recomputed += 1
            seen.add(s["seq_id"])
    assert recomputed > 0
    max_batch, max_tokens, watermark = (int(x) for x in z["sched"])
    blocks = BlockAllocator(int(z["num_blocks"]))
    sched = Scheduler(int(z["block_size"]), max_batch, max_tokens, watermark)
    prompts, max_new = trace_requests(z)
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        sched.add_request(i + 1, p, m)
    preempted = 0
    for st in steps:
        preempted += sched.schedule_step(blocks)["preempted"]
        sched.process_outputs(blocks, st["sampled"])
    assert preempted == sched.counts()["preemptions"] >= recomputed


def test_scheduler_edge_rules():
    """Empty prompt -> {1}; max_new 0 -> 1; the first admission into an empty
    batch ignores the token budget; the watermark holds back admission; EOS
    retires a sequence early."""
    from nvllm.host import BlockAllocator, Scheduler
    blocks = BlockAllocator(10)
    s = Scheduler(4, max_batch_size=4, max_tokens_per_step=3, watermark_blocks=2)
    s.add_request(1, [], 0)                   # becomes [1], max_new 1
    s.add_request(2, list(range(1, 11)), 5)   # 10 tokens > budget 3
    s.schedule_step(blocks)
    rec = s.batch_record(0)
    assert rec[:3].tolist() == [-1, 0, 1] and rec[3:8].tolist() == [1, 0, 1, 1, 1]
    assert s.process_outputs(blocks, [7]) == 1  # max_new 1: retired at once
    sm = s.schedule_step(blocks)  # seq 2 alone: budget exempt, 3 blocks + 2 watermark <= 10
    assert sm["admitted"] == 1 and sm["scheduled_tokens"] == 10
    # watermark: 7 free, a 24-token prompt needs 6 blocks + 2 spare > 7
    s.add_request(3, list(range(1, 25)), 2)
    s.process_outputs(blocks, [9])
    sm = s.schedule_step(blocks)
    assert sm["admitted"] == 0 and sm["batch_size"] == 1
    s2 = Scheduler(4, max_batch_size=2, max_tokens_per_step=64, watermark_blocks=0,
                   eos_token_id=42)
    b2 = BlockAllocator(8)
    s2.add_request(1, [5, 6], 10)
    s2.schedule_step(b2)
    assert s2.process_outputs(b2, [42]) == 1
    assert b2.num_free() == 8
