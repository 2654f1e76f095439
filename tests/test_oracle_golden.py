"""Pins the C oracle against the reference's own outputs (CPU only).

The golden fixtures were produced by the reference's PagedKVCache and
TransformerModel::forward_batch (see tests/golden/make_golden.py). The oracle
must reproduce the slot mapping bit-exactly and the attention output within
TOL_ORACLE (the reference is built with -O3 -ffast-math, which reorders its
dot products, so a few ulp of difference are expected).
"""
import numpy as np
import pytest

from casegen import det_ints, make_case
from helpers import TOL_ORACLE, golden_case, golden_names, load_golden, oracle_run


@pytest.mark.parametrize("name", golden_names())
def test_case_inputs_match_fixture(name):
    case = golden_case(name)
    g = load_golden(name)
    assert np.array_equal(g["num_computed"], case.num_computed)
    assert np.array_equal(g["total_len"], case.total_len)
    assert np.array_equal(g["block_tables"], case.block_tables)
    ck = case.checksums()
    np.testing.assert_allclose(g["checksums"], [ck[k] for k in ("hist_k", "hist_v", "q", "k", "v")],
                               rtol=0, atol=1e-6)


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(oracle, name):
    case = golden_case(name)
    g = load_golden(name)
    ka, va, out, md = oracle_run(oracle, case)
    assert np.array_equal(md["slots"], g["slot_mapping"]), "slot mapping must be bit-exact"
    err = np.abs(out - g["attn_out"]).max()
    assert err <= TOL_ORACLE, f"oracle vs reference max-abs {err}"
    # every new token's K/V row sits where the reference wrote it
    B = case.block_size
    for t, slot in enumerate(md["slots"]):
        for layer in range(case.num_layers):
            assert np.array_equal(ka[slot // B, layer, slot % B], case.k[layer, t])
            assert np.array_equal(va[slot // B, layer, slot % B], case.v[layer, t])


@pytest.mark.parametrize("name", golden_names())
def test_oracle_f64_agrees(oracle, name):
    """The float oracle stays within 2e-6 of a double-precision evaluation."""
    case = golden_case(name)
    _, _, out32, _ = oracle_run(oracle, case)
    _, _, out64, _ = oracle_run(oracle, case, use_f64=True)
    assert np.abs(out32 - out64).max() < 2e-6


def test_flatten_matches_reference_rules(oracle):
    """src/model.cpp:144-157: sequence-major, positions num_computed.., last index."""
    fl = oracle.flatten(np.array([0, 3, 9], np.int32), np.array([4, 4, 12], np.int32))
    assert fl["cu_seqlens_q"].tolist() == [0, 4, 5, 8]
    assert fl["positions"].tolist() == [0, 1, 2, 3, 3, 9, 10, 11]
    assert fl["seq_of_token"].tolist() == [0, 0, 0, 0, 1, 2, 2, 2]
    assert fl["last_token_idx"].tolist() == [3, 4, 7]
    assert fl["context_lens"].tolist() == [4, 4, 12]


def test_reshape_skips_negative_slots(oracle):
    from oracle.oracle import KVLayout
    lay = KVLayout(4, 1, 2, 1, 4)
    ka = np.zeros((4, 1, 2, 4), np.float32)
    va = np.zeros_like(ka)
    k = np.arange(8, dtype=np.float32).reshape(2, 4)
    oracle.reshape_and_cache(k, -k, ka, va, np.array([-1, 5], np.int32), 0, lay)
    assert np.array_equal(ka[2, 0, 1], k[1]) and np.array_equal(va[2, 0, 1], -k[1])
    assert np.count_nonzero(ka) == 4  # only k[1] = [4,5,6,7]; nothing for slot -1


def test_reference_harness_agrees_on_random_cases(oracle):
    """Where the reference build exists (it is built from the reference
    sources), cross-check the oracle on extra seeded cases."""
    from oracle.oracle import KVLayout, RefPath, reference_available
    if not reference_available():
        pytest.skip("reference harness not built here")
    ref = RefPath()
    for seed in range(3):
        S = 5
        total = det_ints(900 + seed, 1, S, 1, 90)
        comp = np.minimum(total - 1, det_ints(900 + seed, 2, S, 0, 90))
        case = make_case(f"rand{seed}", 900 + seed, num_heads=4, head_dim=32,
                         block_size=[2, 4, 16][seed], num_layers=2, num_computed=comp,
                         total_len=total)
        lay = KVLayout(case.num_blocks, case.num_layers, case.block_size, case.num_heads,
                       case.head_dim)
        c = ref.cache_create(lay)
        eng = ref.engine_create(case.num_layers, case.num_heads, case.head_dim, 2)
        bt64 = case.block_tables.astype(np.int64)
        ref.write_history(c, case.num_computed, bt64, case.hist_k, case.hist_v)
        out = np.zeros((case.num_layers, case.n_tokens, case.hidden), np.float32)
        ref.forward_attention(eng, c, case.q_lens, case.total_len, bt64, case.q, case.k, case.v,
                              out)
        ref.cache_destroy(c)
        _, _, out_o, _ = oracle_run(oracle, case)
        assert np.abs(out - out_o).max() <= TOL_ORACLE
