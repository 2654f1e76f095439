"""The HTTP/SSE front end (nvllm_server_*) over the router on the GPU: the
reference server's routes and wire format (src/server.cpp:114-209) with the
reference's own configuration (src/main.cpp: toy model, 1024 blocks of 16,
batch 32, 512 tokens per step, watermark 4).

* GET /health answers OK; unknown paths 404;
* POST /v1/generate streams one SSE frame per generated token, the first with
  ttft_us, the last with finished true, the text the reference model's
  vocabulary string of the token; several clients at once;
* every stream's token ids equal those of the same prompt (tokenised as the
  reference's engine does) generated directly by a Generator on the same model;
* GET /v1/metrics is the reference's MetricsSnapshot JSON summed over the GPUs
  with a per-GPU list.
"""
import http.client
import json
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOY = dict(vocab=512, hidden=128, layers=2, heads=4, head_dim=32, ffn=256)
WORDS = ["system", "kernel", "cpp26", "batch", "token", "cache", "paged", "memory", "tensor",
         "matrix", "stream", "async", "latency", "throughput", "compute", "sched"]
PROMPTS = ["paged attention on blackwell", "continuous batching with a router",
           "cpp26 kernel stream", "", "one two three four five six seven eight nine ten",
           "tensor memory accelerator"]


def _lanes(n):
    import torch

    import nvllm
    from nvllm.host import Engine, Generator, Model
    lay = nvllm.KVLayout(1024, TOY["layers"], 16, TOY["heads"], TOY["head_dim"])
    gpus = torch.cuda.device_count()
    objs = []
    for i in range(n):
        eng = Engine(lay, max_seqs=32, max_tokens=512, max_blocks_per_seq=64, device=i % gpus)
        model = Model(TOY, eng)
        gen = Generator(eng, model, 32, 512, 4)
        objs.append((eng, model, gen))
    return objs


def _close(objs):
    for eng, model, gen in objs:
        gen.close()
        model.close()
        eng.close()


def _generate(port, prompt, max_tokens):
    conn = http.client.HTTPConnection("127.0.0.1", port, timeout=60)
    body = json.dumps({"prompt": prompt, "max_tokens": max_tokens})
    conn.request("POST", "/v1/generate", body=body,
                 headers={"Content-Type": "application/json"})
    r = conn.getresponse()
    assert r.status == 200 and r.getheader("Content-Type") == "text/event-stream"
    frames = []
    for raw in r.read().decode().split("\n\n"):
        if raw.startswith("data: "):
            frames.append(json.loads(raw[len("data: "):]))
    conn.close()
    return frames


def test_server_streams_the_generator_tokens():
    from nvllm.host import Router, Server, tokenize_prompt
    lanes = _lanes(2)
    try:
        router = Router([g for _, _, g in lanes])
        server = Server(router, TOY["vocab"])
        try:
            c = http.client.HTTPConnection("127.0.0.1", server.port, timeout=30)
            c.request("GET", "/health")
            r = c.getresponse()
            assert r.status == 200 and r.read() == b"OK"
            c.close()
            c = http.client.HTTPConnection("127.0.0.1", server.port, timeout=30)
            c.request("GET", "/nope")
            assert c.getresponse().status == 404
            c.close()

            results = {}

            def client(i, prompt):
                results[i] = _generate(server.port, prompt, 8 + 3 * i)

            threads = [threading.Thread(target=client, args=(i, p)) for i, p in enumerate(PROMPTS)]
            for t in threads:
                t.start()
            for t in threads:
                t.join(timeout=120)
            assert len(results) == len(PROMPTS)
            seq_ids = set()
            for i, frames in results.items():
                assert len(frames) == 8 + 3 * i
                assert "ttft_us" in frames[0] and frames[0]["ttft_us"] >= 0
                assert all("ttft_us" not in f for f in frames[1:])
                assert [f["finished"] for f in frames] == [False] * (len(frames) - 1) + [True]
                assert len({f["seq_id"] for f in frames}) == 1
                seq_ids.add(frames[0]["seq_id"])
                for f in frames:
                    assert f["text"] == " " + WORDS[f["token_id"] % 16]
            assert len(seq_ids) == len(PROMPTS)

            c = http.client.HTTPConnection("127.0.0.1", server.port, timeout=30)
            c.request("GET", "/v1/metrics")
            m = json.loads(c.getresponse().read())
            c.close()
            assert m["total_requests_completed"] == len(PROMPTS)
            assert m["total_tokens_generated"] == sum(8 + 3 * i for i in range(len(PROMPTS)))
            assert len(m["gpus"]) == 2
            assert sum(g["requests_completed"] for g in m["gpus"]) == len(PROMPTS)
            assert m["kv_cache_used_blocks"] == 0 and m["active_batch_size"] == 0
        finally:
            server.close()
            router.close()
    finally:
        _close(lanes)

    # the same prompts straight through one generator on the same model
    solo = _lanes(1)
    try:
        _, _, gen = solo[0]
        for i, p in enumerate(PROMPTS):
            gen.add_request(i + 1, tokenize_prompt(p, TOY["vocab"]), 8 + 3 * i)
        gen.run()
        for i, p in enumerate(PROMPTS):
            toks = tokenize_prompt(p, TOY["vocab"])
            want = gen.output(i + 1)[len(toks):].tolist()
            assert [f["token_id"] for f in results[i]] == want, f"prompt {i}"
    finally:
        _close(solo)
