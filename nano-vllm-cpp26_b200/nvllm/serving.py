"""Serving workloads for the generator (scheduler + engine + device model) and
the sizing of an engine for them.

* ``serve_toy``: the reference's own continuous-batching benchmark
  (src/benchmark.cpp:46-67, :238-261): the toy model (vocab 512, d 128, 2
  layers, 4 heads of 32, ffn 256), 1024 blocks of 16, batch 16, 512 tokens per
  step, watermark 2, 96 requests from its deterministic generator (prompt
  8 + i % 12 tokens, 128 new tokens when i % 5 == 0, else 16).
* ``serve_toy_seeded``: the same with seeded prompts of uniform length 8-32
  and uniform token ids, 20 % of the requests asking for 128 tokens.
* ``longctx_model``: long-context decode inside the 4096-wide model: 4
  requests of 32768 seeded prompt tokens each (the long-context attention
  workload's shape), one prompt per step beside the running decodes, then
  decode; with head parallelism every rank holds heads / N of every sequence.
* ``serve``: the 4096-wide model (32 heads of 128, ffn 11008, 4 layers, vocab
  32000, LCG weights) under a serving load: prompt lengths lognormal with
  median 256 (sigma 1.0, at most 4096 tokens), completions 16 tokens for 80 %
  of the requests and 512 for 20 %, batch 256; 128 requests per GPU, so that 8
  GPUs serve 1024. Seeded synthetic prompts stand in for real text.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

TOY_MODEL = dict(vocab=512, hidden=128, layers=2, heads=4, head_dim=32, ffn=256)
WIDE_MODEL = dict(vocab=32000, hidden=4096, layers=4, heads=32, head_dim=128, ffn=11008)


@dataclass
class ServeSpec:
    name: str
    model: dict
    num_blocks: int
    block_size: int
    max_batch: int
    max_tokens_per_step: int
    watermark: int
    prompts: list = field(default_factory=list)
    max_new: list = field(default_factory=list)

    @property
    def longest(self) -> int:
        return max(len(p) + m for p, m in zip(self.prompts, self.max_new))

    @property
    def output_tokens(self) -> int:
        return int(sum(self.max_new))

    @property
    def prompt_tokens(self) -> int:
        return int(sum(len(p) for p in self.prompts))

    def engine_limits(self) -> dict:
        """max_seqs / max_tokens / max_blocks_per_seq that hold any step of this
        workload: a step carries at most max(token budget, the longest
        sequence recomputed alone, one decode token per running sequence)."""
        longest = self.longest
        return dict(max_seqs=self.max_batch,
                    max_tokens=max(self.max_tokens_per_step, longest, self.max_batch),
                    max_blocks_per_seq=(longest + self.block_size - 1) // self.block_size)


def bimodal_requests(n: int, vocab: int):
    """src/benchmark.cpp:46-67."""
    prompts = [[((i * 31 + j * 17) % (vocab - 1)) + 1 for j in range(8 + i % 12)]
               for i in range(n)]
    return prompts, [128 if i % 5 == 0 else 16 for i in range(n)]


def seeded_toy_requests(n: int, vocab: int, seed: int):
    rng = np.random.default_rng(seed)
    lens = rng.integers(8, 33, n)
    prompts = [rng.integers(1, vocab, int(k)).tolist() for k in lens]
    max_new = np.where(rng.random(n) < 0.2, 128, 16).tolist()
    return prompts, max_new


def lognormal_requests(n: int, vocab: int, seed: int, median: int = 256, sigma: float = 1.0,
                       cap: int = 4096):
    rng = np.random.default_rng(seed)
    lens = np.clip(np.rint(np.exp(rng.normal(np.log(median), sigma, n))), 1, cap).astype(int)
    prompts = [rng.integers(1, vocab, int(k)).tolist() for k in lens]
    max_new = np.where(rng.random(n) < 0.2, 512, 16).tolist()
    return prompts, max_new


def make_serve(name: str, seed: int = 0, requests: int | None = None) -> ServeSpec:
    if name == "serve_toy":
        prompts, max_new = bimodal_requests(requests or 96, TOY_MODEL["vocab"])
        return ServeSpec(name, TOY_MODEL, 1024, 16, 16, 512, 2, prompts, max_new)
    if name == "serve_toy_seeded":
        prompts, max_new = seeded_toy_requests(requests or 96, TOY_MODEL["vocab"], seed)
        return ServeSpec(name, TOY_MODEL, 1024, 16, 16, 512, 2, prompts, max_new)
    if name == "longctx_model":
        n = requests or 4
        rng = np.random.default_rng(seed)
        prompts = [rng.integers(1, WIDE_MODEL["vocab"], 32768).tolist() for _ in range(n)]
        max_new = [512] * n  # decode runs longer than any timed window
        # a step holds one whole prompt beside the running decodes (the scheduler
        # admits a prompt over the token budget only into an empty batch)
        spec = ServeSpec(name, WIDE_MODEL, 0, 16, n, 32768 + n, 0, prompts, max_new)
        spec.num_blocks = int(sum((len(p) + m + 15) // 16 for p, m in zip(prompts, max_new)) + 16)
        return spec
    if name == "serve":
        prompts, max_new = lognormal_requests(requests or 128, WIDE_MODEL["vocab"], seed)
        spec = ServeSpec(name, WIDE_MODEL, 0, 16, 256, 16384, 4, prompts, max_new)
        # every request resident at once (no preemption): its blocks plus the
        # watermark, rounded up
        need = sum((len(p) + m + 15) // 16 for p, m in zip(prompts, max_new))
        spec.num_blocks = int(need + 64)
        return spec
    raise ValueError(f"unknown serving workload {name}")


def serve_config(spec: ServeSpec) -> dict:
    m = spec.model
    return {"workload": {
        "serve_toy": "reference continuous-batching benchmark (toy model, 96 requests)",
        "serve_toy_seeded": "toy model, 96 seeded requests (prompts U[8,32])",
        "serve": "e2e serving, 4096-wide 4-layer model, 128 requests per GPU",
        "longctx_model": "long-context decode in the 4096-wide model: 4 sequences of 32768 "
                         "prompt tokens, heads split over the GPUs",
    }[spec.name], "model": f"d{m['hidden']} L{m['layers']} H{m['heads']}x{m['head_dim']} "
                          f"ffn{m['ffn']} vocab{m['vocab']} (LCG weights)",
        "requests": len(spec.prompts), "prompt_tokens": spec.prompt_tokens,
        "output_tokens": spec.output_tokens, "max_batch": spec.max_batch,
        "max_tokens_per_step": spec.max_tokens_per_step, "block_size": spec.block_size,
        "num_blocks": spec.num_blocks, "watermark_blocks": spec.watermark}
