"""The generator (scheduler + engine + device model, nvllm_generator_*) end to
end on the GPU against the reference's continuous-batching run: given the same
requests it must write the reference's trace — every step's batch (sequences,
lengths, block tables, uncomputed tokens) and every sampled token identical,
the top-2 margins and top-8 logits within LOGIT_RTOL — and finish every request
with the reference's token stream."""
import json

import numpy as np
import pytest

from helpers import LOGIT_RTOL, load_trace, trace_requests

pytestmark = pytest.mark.gpu


def build(name, precision=0, graph_max_tokens=0, gemm_math=0):
    import nvllm
    from nvllm.host import Engine, Generator, Model
    cfg, z, steps = load_trace(name)
    max_batch, max_tokens, watermark = (int(x) for x in z["sched"])
    lay = nvllm.KVLayout(int(z["num_blocks"]), cfg["layers"], int(z["block_size"]), cfg["heads"],
                         cfg["head_dim"])
    prompts, max_new = trace_requests(z)
    longest = max(len(p) + m for p, m in zip(prompts, max_new))
    B = int(z["block_size"])
    eng = Engine(lay, max_seqs=max_batch, max_tokens=max(max_tokens, longest),
                 max_blocks_per_seq=(longest + B - 1) // B)
    model = Model(cfg, eng, scales=z["scales"][:2], graph_max_tokens=graph_max_tokens,
                  gemm_math=gemm_math)
    gen = Generator(eng, model, max_batch, max_tokens, watermark, precision=precision)
    for i, (p, m) in enumerate(zip(prompts, max_new)):
        gen.add_request(i + 1, p, m)
    return cfg, z, steps, (eng, model, gen), prompts


@pytest.mark.parametrize("gemm,precision", [(0, 0), (2, 0), (2, 1)],
                         ids=["ffma", "tcgen05", "tcgen05-tf32attn"])
@pytest.mark.parametrize("graphs", [0, 512], ids=["eager", "graphs"])
@pytest.mark.parametrize("name", ["tokens_toy_seeded", "tokens_toy_bench", "tokens_wide"])
def test_generator_reproduces_reference_run(name, graphs, gemm, precision, tmp_path):
    """graphs 512: every step of at most 512 new tokens is padded to a
    power-of-two bucket and replayed as that bucket's CUDA graph; gemm 2: every
    projection on this library's GEMMs (tcgen05 above 32 rows, the decode-size
    kernels below); precision 1: the prefill attention tiles on the tcgen05
    kernel (two-term bf16 products) where the geometry has it (the FFMA kernel
    elsewhere)."""
    from nvllm.host import metrics_json
    from oracle.oracle import read_trace
    cfg, z, steps, objs, prompts = build(name, precision=precision, graph_max_tokens=graphs,
                                         gemm_math=gemm)
    eng, model, gen = objs
    try:
        path = str(tmp_path / "run.trace")
        gen.trace(path)
        n_steps = gen.run()
        gen.trace(None)
        assert n_steps == len(steps)
        mine = read_trace(path)
        assert len(mine) == len(steps)
        streams = {i + 1: list(p) for i, p in enumerate(prompts)}
        for i, (a, b) in enumerate(zip(mine, steps)):
            assert np.array_equal(a["record"], b["record"]), f"{name} step {i}: batch"
            assert np.array_equal(a["sampled"], b["sampled"]), f"{name} step {i}: tokens"
            scale = np.abs(b["top_val"]).max(axis=1, keepdims=True)
            assert (np.abs(a["top_val"] - b["top_val"]) <= LOGIT_RTOL * scale).all()
            np.testing.assert_allclose(a["margin"], b["margin"], rtol=0,
                                       atol=2 * LOGIT_RTOL * float(scale.max()))
            for s, t in zip(b["seqs"], b["sampled"]):
                streams[s["seq_id"]].append(int(t))
        for sid, want in streams.items():
            got = gen.output(sid)
            assert got is not None and got.tolist() == want, f"sequence {sid}"
        m = gen.metrics()
        assert m.total_requests_received == m.total_requests_completed == len(prompts)
        assert m.total_tokens_generated == sum(len(st["seqs"]) for st in steps)
        assert m.total_iterations == len(steps)
        assert m.active_batch_size == 0 and m.waiting_queue_depth == 0
        assert m.kv_cache_used_blocks == 0
        snap = json.loads(metrics_json(m))
        assert snap["total_requests_completed"] == len(prompts)
        assert not gen.has_pending_work()
    finally:
        gen.close()
        model.close()
        eng.close()


def test_generator_step_by_step_and_preemption_count():
    """Stepping by hand gives the same summaries as the reference's batches,
    and the tight arena of the seeded run preempts."""
    cfg, z, steps, objs, prompts = build("tokens_toy_seeded")
    eng, model, gen = objs
    try:
        preempted = 0
        for st in steps:
            s = gen.step()
            assert s["batch_size"] == len(st["seqs"])
            preempted += s["preempted"]
        assert not gen.has_pending_work()
        assert preempted > 0 and gen.metrics().total_preemptions == preempted
    finally:
        gen.close()
        model.close()
        eng.close()


@pytest.mark.parametrize("burst", [False, True])
@pytest.mark.parametrize("lanes", [2, 3])
def test_router_serves_every_request_with_the_reference_stream(lanes, burst):
    """The reference benchmark's 96 requests through nvllm_router over several
    generators, each with its own engine (arena, allocator, scheduler), model
    and engine thread: on distinct GPUs where the box has them, else several on
    cuda:0. Every request finishes on the GPU the router chose with the token
    stream the reference produced for it; the requests spread over the lanes by
    outstanding work. Placed one call per request, or as one burst
    (nvllm_router_add_requests), which is all or nothing."""
    import torch

    import nvllm
    from nvllm.host import Engine, Generator, Model, Router
    cfg, z, steps = load_trace("tokens_toy_bench")
    max_batch, max_tokens, watermark = (int(x) for x in z["sched"])
    prompts, max_new = trace_requests(z)
    want = {i + 1: list(p) for i, p in enumerate(prompts)}
    for st in steps:
        for s, t in zip(st["seqs"], st["sampled"]):
            want[s["seq_id"]].append(int(t))
    longest = max(len(p) + m for p, m in zip(prompts, max_new))
    B = int(z["block_size"])
    lay = nvllm.KVLayout(int(z["num_blocks"]), cfg["layers"], B, cfg["heads"], cfg["head_dim"])
    gpus = torch.cuda.device_count()
    objs = []
    try:
        for i in range(lanes):
            eng = Engine(lay, max_seqs=max_batch, max_tokens=max(max_tokens, longest),
                         max_blocks_per_seq=(longest + B - 1) // B, device=i % gpus)
            model = Model(cfg, eng, scales=z["scales"][:2])
            gen = Generator(eng, model, max_batch, max_tokens, watermark)
            objs.append((eng, model, gen))
        router = Router([g for _, _, g in objs])
        try:
            if burst:
                with pytest.raises(nvllm.NvllmError):  # an id repeated in the burst
                    router.add_requests([1, 1], prompts[:2], max_new[:2])
                placed = router.add_requests([i + 1 for i in range(len(prompts))], prompts,
                                             max_new).tolist()
            else:
                placed = [router.add_request(i + 1, p, m)
                          for i, (p, m) in enumerate(zip(prompts, max_new))]
            router.wait_idle()
            assert sorted(set(placed)) == list(range(lanes))
            for lane in range(lanes):
                assert router.placed(lane) == placed.count(lane)
            for sid, stream in want.items():
                got = router.output(sid)
                assert got is not None and got.tolist() == stream, f"sequence {sid}"
            total = 0
            for lane in range(lanes):
                m = router.metrics(lane)
                assert m.total_requests_received == m.total_requests_completed
                assert m.total_requests_completed == placed.count(lane)
                assert m.active_batch_size == 0 and m.kv_cache_used_blocks == 0
                total += m.total_tokens_generated
            assert total == sum(max_new)
            with pytest.raises(nvllm.NvllmError):
                router.add_request(1, prompts[0], 4)  # id already used
        finally:
            router.close()
    finally:
        for eng, model, gen in objs:
            gen.close()
            model.close()
            eng.close()
