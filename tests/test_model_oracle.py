"""The model oracle (oracle/model.py) pinned against the reference:

* the LCG jump-ahead equals the reference's sequential generator;
* the weights equal, bit for bit, the W operands the reference's own
  forward_batch hands to matmul_batched;
* replaying the reference's token traces (scheduler + forward_batch, real
  matmuls) through the oracle reproduces every sampled token and the top-8
  LM-head logits.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import LOGIT_RTOL, load_trace
from oracle import model as M
from oracle.oracle import reference_available

TRACES = ("tokens_toy_seeded", "tokens_toy_bench")


def sequential_draws(offset: int, count: int, scale: np.float32) -> np.ndarray:
    """The reference constructor's next_f32 loop (src/model.cpp:71-79), run
    draw by draw."""
    seed = M.SEED
    out = np.zeros(count, np.float32)
    for i in range(offset + count):
        seed = (seed * M.MUL + 1) & M.MASK
        if i >= offset:
            unit = np.float32(seed >> 33) / np.float32(4294967296.0) - np.float32(0.5)
            out[i - offset] = unit * scale
    return out


@pytest.mark.parametrize("offset,count", [(0, 1), (0, 100), (37, 64), (1000, 333)])
def test_lcg_jump_ahead_matches_sequential(offset, count):
    sc = np.float32(0.08838834)
    assert np.array_equal(M.lcg_draws(offset, count, sc), sequential_draws(offset, count, sc))


def test_weight_offsets_cover_the_stream():
    cfg = dict(vocab=10, hidden=4, layers=2, heads=2, head_dim=2, ffn=6)
    off = M.weight_offsets(cfg)
    per_layer = 4 * 16 + 2 * 24
    assert off[(0, "w_q")] == 40
    assert off[(1, "w_q")] == 40 + per_layer
    assert off[(1, "w_down")] == 40 + per_layer + 4 * 16 + 24
    assert off["lm_head"] == 40 + 2 * per_layer
    assert off["total"] == off["lm_head"] + 40


@pytest.mark.skipif(not reference_available(), reason="reference harness not built")
def test_weights_bit_exact_against_reference_operands():
    from casegen import TOY_MODEL
    from oracle.oracle import RefPath
    ref = RefPath()
    scales = ref.model_scales(TOY_MODEL)
    ops = ref.model_operands(TOY_MODEL, 7)
    assert len(ops) == 6 * TOY_MODEL["layers"] + 1
    w = M.model_weights(TOY_MODEL, scales)
    names = ("w_q", "w_k", "w_v", "w_o", "w_up", "w_down")
    for i, (a, wt) in enumerate(ops):
        mine = w["layers"][i // 6][names[i % 6]] if i < len(ops) - 1 else w["lm_head"]
        assert np.array_equal(mine, wt), f"matmul call {i}"
    # the first A operand is the RMSNorm of the token's embedding row
    np.testing.assert_allclose(ops[0][0], M.rms_norm(w["embedding"][[7]]), rtol=0, atol=1e-6)


@pytest.mark.skipif(not reference_available(), reason="reference harness not built")
def test_fixture_scales_are_the_reference_builds():
    from oracle.oracle import RefPath
    ref = RefPath()
    for name in TRACES + ("tokens_wide",):
        cfg, z, _ = load_trace(name)
        assert np.array_equal(z["scales"], ref.model_scales(cfg))
        # within one unit in the last place of the correctly rounded values
        d = np.abs(z["scales"].view(np.int32) - M.default_scales(cfg).view(np.int32))
        assert (d <= 1).all()


@pytest.mark.parametrize("name", TRACES)
def test_oracle_replays_reference_token_trace(name):
    cfg, z, steps = load_trace(name)
    mo = M.ModelOracle(cfg, int(z["num_blocks"]), int(z["block_size"]), scales=z["scales"])
    assert len(steps) > 0
    for i, st in enumerate(steps):
        sampled, margin, logits = mo.forward(st["seqs"])
        assert np.array_equal(sampled, st["sampled"]), f"step {i}"
        got = np.take_along_axis(logits, st["top_idx"], axis=1)
        scale = np.abs(st["top_val"]).max(axis=1, keepdims=True)
        assert (np.abs(got - st["top_val"]) <= LOGIT_RTOL * scale).all(), f"step {i}"
        np.testing.assert_allclose(margin, st["margin"], rtol=0, atol=LOGIT_RTOL * scale.max())


def test_trace_is_self_consistent():
    """Each step's sampled token becomes the sequence's last token the next time
    it runs (src/scheduler.cpp process_step_outputs), and every running
    sequence's table covers its total length."""
    cfg, z, steps = load_trace("tokens_toy_seeded")
    B = int(z["block_size"])
    last = {}
    for st in steps:
        for s, tok in zip(st["seqs"], st["sampled"]):
            assert len(s["table"]) * B >= s["total_len"]
            assert s["total_len"] - s["num_computed"] == len(s["uncomputed"])
            if s["seq_id"] in last and s["num_computed"] > 0:
                assert s["prev_token"] == last[s["seq_id"]]
            last[s["seq_id"]] = int(tok)


def test_penalized_argmax_rules():
    logits = np.array([[1.0, 3.0, 3.0, 2.0],
                       [5.0, 4.0, 4.0, 0.0],
                       [0.0, 0.0, 0.0, 0.0]], np.float32)
    prev = np.array([9, 0, 3], np.int64)  # 9: outside the vocabulary, no penalty
    sampled, margin = M.penalized_argmax(logits, prev)
    assert sampled.tolist() == [1, 1, 0]  # first maximum wins ties
    np.testing.assert_array_equal(margin, np.array([0.0, 0.0, 0.0], np.float32))
    sampled, margin = M.penalized_argmax(logits[:1], np.array([1], np.int64))
    assert sampled.tolist() == [2]
    assert margin[0] == np.float32(1.0)
