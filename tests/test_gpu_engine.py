"""The host engine (libnvllm_host.so) end to end on the GPU: metadata packed
and uploaded by the engine, host Q/K/V rows in, attention rows out, against the
reference's golden outputs. Iteration 1 writes each sequence's cached history
through the engine itself (a prefill with the history rows); iteration 2 is
the golden step."""
import numpy as np
import pytest

from helpers import TOL_FP32, TOL_TF32, golden_case, load_golden

pytestmark = pytest.mark.gpu


def _tables(case):
    nb = (case.total_len + case.block_size - 1) // case.block_size
    return [case.block_tables[s, :nb[s]] for s in range(len(case.total_len))]


def run_engine(case, precision=0, use_pinned=False):
    import nvllm
    from nvllm.host import Engine
    lay = nvllm.KVLayout(case.num_blocks, case.num_layers, case.block_size, case.num_heads,
                         case.head_dim)
    n_hist = int(case.num_computed.sum())
    max_tokens = max(n_hist, case.n_tokens, 1)
    eng = Engine(lay, max_seqs=len(case.total_len), max_tokens=max_tokens,
                 max_blocks_per_seq=case.block_tables.shape[1], device=0)
    tables = _tables(case)
    try:
        if n_hist:
            eng.begin_step(np.zeros_like(case.num_computed), case.num_computed, tables)
            assert eng.step_tokens() == n_hist
            junk = np.zeros((n_hist, case.hidden), np.float32)
            for layer in range(case.num_layers):
                eng.attention(layer, junk, case.hist_k[layer], case.hist_v[layer], junk.copy())
        eng.begin_step(case.num_computed, case.total_len, tables)
        assert eng.step_tokens() == case.n_tokens
        outs = []
        for layer in range(case.num_layers):
            if use_pinned:
                n = case.n_tokens
                q, k, v, o = (p[:n] for p in eng.pinned)
                q[:] = case.q[layer]
                k[:] = case.k[layer]
                v[:] = case.v[layer]
                eng.attention(layer, q, k, v, o, precision)
                outs.append(o.copy())
            else:
                out = np.full((case.n_tokens, case.hidden), np.nan, np.float32)
                eng.attention(layer, np.ascontiguousarray(case.q[layer]),
                              np.ascontiguousarray(case.k[layer]),
                              np.ascontiguousarray(case.v[layer]), out, precision)
                outs.append(out)
        assert nvllm.get_last_error(eng.stream()) == nvllm.OK
        return np.stack(outs)
    finally:
        eng.close()


@pytest.mark.parametrize("name", ["decode_h4_hd32_b16", "mixed_h4_hd32_b4", "mixed_h32_hd128_b16",
                                  "decode_h32_hd128_b16", "mixed_h8_hd64_b16"])
def test_engine_matches_golden(name):
    case = golden_case(name)
    g = load_golden(name)
    out = run_engine(case)
    err = np.abs(out - g["attn_out"]).max()
    assert err <= TOL_FP32, f"{name}: engine vs reference max-abs {err}"


def test_engine_pinned_rows_and_tf32():
    case = golden_case("mixed_h32_hd128_b16")
    g = load_golden(case.name)
    out = run_engine(case, precision=1, use_pinned=True)
    assert np.abs(out - g["attn_out"]).max() <= TOL_TF32


def test_engine_allocator_and_errors():
    import nvllm
    from nvllm.host import Engine
    lay = nvllm.KVLayout(8, 1, 4, 2, 32)
    eng = Engine(lay, max_seqs=2, max_tokens=8, max_blocks_per_seq=4)
    try:
        ids = eng.allocate_blocks(5)
        assert ids.tolist() == [0, 1, 2, 3, 4] and eng.num_free() == 3
        assert eng.allocate_blocks(4) is None
        assert eng.free_blocks(ids) == 0 and eng.num_free() == 8
        with pytest.raises(nvllm.NvllmError):   # 9 tokens > max_tokens 8
            eng.begin_step([0], [9], [[0, 1, 2]])
        with pytest.raises(nvllm.NvllmError):   # table too short
            eng.begin_step([0], [8], [[0]])
    finally:
        eng.close()


@pytest.mark.parametrize("name", ["mixed_h4_hd32_b4", "mixed_h32_hd128_b16"])
def test_engine_pipelined_slots_match_golden(name):
    """The two-slot pipeline (nvllm_engine_attention_submit / _collect): the
    step's layers go alternately to slots 0 and 1, each slot collected only
    before its reuse, so one layer's copies overlap the other's kernels; every
    layer's output equals the reference's. A busy slot and the synchronous
    path are refused while a slot is in flight."""
    import nvllm
    from nvllm.host import Engine
    case = golden_case(name)
    g = load_golden(name)
    lay = nvllm.KVLayout(case.num_blocks, case.num_layers, case.block_size, case.num_heads,
                         case.head_dim)
    n_hist = int(case.num_computed.sum())
    eng = Engine(lay, max_seqs=len(case.total_len), max_tokens=max(n_hist, case.n_tokens, 1),
                 max_blocks_per_seq=case.block_tables.shape[1], device=0)
    tables = _tables(case)
    try:
        if n_hist:
            eng.begin_step(np.zeros_like(case.num_computed), case.num_computed, tables)
            junk = np.zeros((n_hist, case.hidden), np.float32)
            for layer in range(case.num_layers):
                eng.attention(layer, junk, case.hist_k[layer], case.hist_v[layer], junk.copy())
        eng.begin_step(case.num_computed, case.total_len, tables)
        n = case.n_tokens
        slots = [eng.slot_pinned(0), eng.slot_pinned(1)]
        outs = [None] * case.num_layers
        pending = []  # (slot, layer)
        for rep in range(2):  # the layers twice: slots reused across the step
            for layer in range(case.num_layers):
                slot = (rep * case.num_layers + layer) % 2
                for s_, lay_ in list(pending):
                    if s_ == slot:
                        eng.collect(s_)
                        outs[lay_] = slots[s_][3][:n].copy()
                        pending.remove((s_, lay_))
                q, k, v, o = slots[slot]
                q[:n], k[:n], v[:n] = case.q[layer], case.k[layer], case.v[layer]
                o[:n] = np.nan
                eng.submit(layer, slot, 0)
                pending.append((slot, layer))
                with pytest.raises(nvllm.NvllmError):
                    eng.submit(layer, slot, 0)  # in flight
                with pytest.raises(nvllm.NvllmError):
                    eng.attention(layer, q[:n], k[:n], v[:n], o[:n].copy())
        for s_, lay_ in pending:
            eng.collect(s_)
            outs[lay_] = slots[s_][3][:n].copy()
        with pytest.raises(nvllm.NvllmError):
            eng.collect(0)  # nothing in flight
        assert nvllm.get_last_error(eng.stream()) == nvllm.OK
        err = np.abs(np.stack(outs) - g["attn_out"]).max()
        assert err <= TOL_FP32, f"{name}: pipelined engine vs reference max-abs {err}"
    finally:
        eng.close()
