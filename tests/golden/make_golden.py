"""Generates the golden fixtures in this folder by running the reference's own
C++ (PagedKVCache + TransformerModel::forward_batch, built by
``make -C oracle ref`` from the reference sources) on the deterministic cases
of ``tests/casegen.py``.

Run from the repository root, with ``NVLLM_REFERENCE_DIR`` naming a checkout of
the reference:  NVLLM_REFERENCE_DIR=<checkout> python tests/golden/make_golden.py

Each ``<case>.npz`` holds the case description (geometry, per-sequence
num_computed / total_len, block tables), checksums of the generated inputs,
the slot mapping of every new token, and the reference attention output
[L, n_tok, D]. The slot mapping is confirmed against the reference arena: the
K and V rows of each new token are read back through read_head_kv at
(block_table[pos / B], layer, pos % B) and must equal the inputs bit for bit.

``allocator_trace.npz`` records a seeded sequence of allocate_block /
allocate_blocks / free_blocks calls on the reference PagedKVCache with the
block ids and free counts it returned.

``tokens_*.npz`` are traces of the reference's continuous-batching loop
(ContinuousScheduler + TransformerModel::forward_batch with its real matmuls and
LCG weights; see ref_generate in oracle/ref_harness.cpp): every step's running
sequences (computed / total lengths, block tables, uncomputed token ids, the
previous token), the tokens the reference sampled for them, the top-2 margin
of the penalised logits and the 8 largest logits of each sampled row, plus the
reference build's weight and softmax scales (``scales``: 1/sqrt of hidden, ffn
and head_dim as its -ffast-math code evaluates them), the requests
(``prompt_lens``, ``prompt_tokens``, ``max_new``; sequence i + 1 is request i)
and the scheduler settings (``sched``: max_batch, max_tokens_per_step,
watermark_blocks).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from casegen import det_ints, det_uniform, golden_cases  # noqa: E402
from oracle.oracle import KVLayout, RefPath, build  # noqa: E402

OUT = Path(__file__).resolve().parent


def run_case(ref: RefPath, case) -> dict:
    lay = KVLayout(case.num_blocks, case.num_layers, case.block_size, case.num_heads,
                   case.head_dim)
    cache = ref.cache_create(lay)
    eng = ref.engine_create(case.num_layers, case.num_heads, case.head_dim, 4)
    bt64 = case.block_tables.astype(np.int64)
    ref.write_history(cache, case.num_computed, bt64, case.hist_k, case.hist_v)
    n = case.n_tokens
    out = np.zeros((case.num_layers, n, case.hidden), np.float32)
    got = ref.forward_attention(eng, cache, case.q_lens, case.total_len, bt64, case.q, case.k,
                                case.v, out)
    assert got == n
    B = case.block_size
    slots = np.zeros(n, np.int32)
    t = 0
    for s in range(len(case.total_len)):
        for pos in range(int(case.num_computed[s]), int(case.total_len[s])):
            blk = int(case.block_tables[s, pos // B])
            slots[t] = blk * B + pos % B
            for layer in range(case.num_layers):
                for h in range(case.num_heads):
                    kr, vr = ref.read_head_kv(cache, blk, layer, pos % B, h, case.head_dim)
                    sl = slice(h * case.head_dim, (h + 1) * case.head_dim)
                    assert np.array_equal(kr, case.k[layer, t, sl])
                    assert np.array_equal(vr, case.v[layer, t, sl])
            t += 1
    ref.cache_destroy(cache)
    ck = case.checksums()
    return dict(
        name=np.array(case.name), seed=np.int64(case.seed), num_blocks=np.int64(case.num_blocks),
        num_layers=np.int32(case.num_layers), block_size=np.int32(case.block_size),
        num_heads=np.int32(case.num_heads), head_dim=np.int32(case.head_dim),
        num_computed=case.num_computed, total_len=case.total_len,
        block_tables=case.block_tables, slot_mapping=slots, attn_out=out,
        checksums=np.array([ck[k] for k in ("hist_k", "hist_v", "q", "k", "v")]),
    )


def allocator_trace(ref: RefPath, seed: int = 7, num_blocks: int = 40, n_ops: int = 400) -> dict:
    """Seeded allocate/free sequence on the reference allocator
    (src/kv_cache.cpp:23-55)."""
    lay = KVLayout(num_blocks, 1, 4, 1, 4)
    cache = ref.cache_create(lay)
    kinds = det_ints(seed, 1, n_ops, 0, 2)
    counts = det_ints(seed, 2, n_ops, 0, 9)
    picks = det_uniform(seed, 3, n_ops)
    held: list[int] = []
    op_kind, op_arg, results, free_after = [], [], [], []
    for i in range(n_ops):
        kind = int(kinds[i])
        if kind == 0:  # allocate_block
            r = ref.allocate_block(cache)
            op_kind.append(0)
            op_arg.append(1)
            results.append([] if r is None else [r])
            if r is not None:
                held.append(int(r))
        elif kind == 1:  # allocate_blocks(count)
            c = int(counts[i])
            r = ref.allocate_blocks(cache, c)
            op_kind.append(1)
            op_arg.append(c)
            results.append(None if r is None else [int(x) for x in r])
            if r is not None:
                held.extend(int(x) for x in r)
        else:  # free_blocks of a contiguous run of held ids
            if not held:
                op_kind.append(2)
                op_arg.append(0)
                results.append([])
            else:
                start = int(picks[i] * len(held))
                c = max(1, min(int(counts[i]), len(held) - start))
                ids = held[start:start + c]
                del held[start:start + c]
                ref.free_blocks(cache, np.array(ids, np.int64))
                op_kind.append(2)
                op_arg.append(c)
                results.append(ids)
        free_after.append(ref.num_free(cache))
    ref.cache_destroy(cache)
    ok = np.array([r is not None for r in results], np.uint8)
    flat = np.array([x for r in results if r is not None for x in r], np.int64)
    lens = np.array([0 if r is None else len(r) for r in results], np.int32)
    return dict(num_blocks=np.int64(num_blocks), op_kind=np.array(op_kind, np.int32),
                op_arg=np.array(op_arg, np.int32), ok=ok, result_ids=flat, result_lens=lens,
                free_after=np.array(free_after, np.int64))


TOKEN_TRACES = {
    # the reference benchmark's own workload and configuration
    # (src/benchmark.cpp:46-67, :238-261): toy model, 96 requests, batch 16
    "tokens_toy_bench": dict(model="toy", num_blocks=1024, block_size=16, max_batch=16,
                             max_tokens_per_step=512, watermark=2, requests="bench"),
    # seeded prompts of 8-32 tokens, block size 8, a tight arena that forces
    # preemption by recompute (src/scheduler.cpp:44-76)
    "tokens_toy_seeded": dict(model="toy", num_blocks=48, block_size=8, max_batch=12,
                              max_tokens_per_step=256, watermark=1, requests="seeded"),
    # the 4096-hidden, 32-head, 4-layer, vocab-32000 model of the serving workload
    "tokens_wide": dict(model="wide", num_blocks=64, block_size=16, max_batch=4,
                        max_tokens_per_step=512, watermark=0, requests="wide"),
}


def token_requests(kind: str):
    from casegen import TOY_MODEL, bimodal_workload
    if kind == "bench":
        return bimodal_workload(96, TOY_MODEL["vocab"])
    if kind == "seeded":
        lens = det_ints(11, 1, 24, 8, 32)
        toks = det_ints(11, 2, int(lens.sum()), 1, TOY_MODEL["vocab"] - 1)
        prompts, off = [], 0
        for n in lens:
            prompts.append(toks[off:off + n].tolist())
            off += int(n)
        max_new = [int(x) for x in det_ints(11, 3, 24, 4, 40)]
        return prompts, max_new
    prompts = [[int(x) for x in det_ints(12, i, n, 1, 31999)] for i, n in enumerate((12, 7, 20))]
    return prompts, [3, 2, 3]


def token_trace(ref: RefPath, spec: dict) -> dict:
    import tempfile

    from casegen import TOY_MODEL, WIDE_MODEL
    model = TOY_MODEL if spec["model"] == "toy" else WIDE_MODEL
    prompts, max_new = token_requests(spec["requests"])
    with tempfile.NamedTemporaryFile(suffix=".trace") as f:
        ref.generate(model, spec["num_blocks"], spec["block_size"], spec["max_batch"],
                     spec["max_tokens_per_step"], spec["watermark"], prompts, max_new, f.name)
        raw = np.fromfile(f.name, dtype="<i8")
    # float bit patterns are uint32: keep the trace as int64
    return dict(trace=raw, model=np.array([model[k] for k in
                ("vocab", "hidden", "layers", "heads", "head_dim", "ffn")], np.int64),
                num_blocks=np.int64(spec["num_blocks"]), block_size=np.int64(spec["block_size"]),
                scales=ref.model_scales(model),
                sched=np.array([spec["max_batch"], spec["max_tokens_per_step"],
                                spec["watermark"]], np.int64),
                prompt_lens=np.array([len(p) for p in prompts], np.int64),
                prompt_tokens=np.concatenate([np.asarray(p, np.int64) for p in prompts]),
                max_new=np.asarray(max_new, np.int64))


def main() -> None:
    import sys
    build(with_reference=True)
    ref = RefPath()
    if "--tokens-only" not in sys.argv:
        _main_cases(ref)
    for name, spec in TOKEN_TRACES.items():
        np.savez_compressed(OUT / f"{name}.npz", **token_trace(ref, spec))
        print(f"{name} saved")


def _main_cases(ref: RefPath) -> None:
    for case in golden_cases():
        data = run_case(ref, case)
        np.savez_compressed(OUT / f"{case.name}.npz", **data)
        print(f"{case.name}: n_tok={case.n_tokens} saved")
    np.savez_compressed(OUT / "allocator_trace.npz", **allocator_trace(ref))
    print("allocator_trace saved")


if __name__ == "__main__":
    main()
