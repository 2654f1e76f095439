"""Host library on the CPU: the block allocator against the reference
allocator's recorded trace, and the metadata packer against the golden slot
mappings / block tables (bit-exact) and the oracle's flatten."""
import numpy as np
import pytest

from casegen import det_ints, golden_cases, make_case
from helpers import load_golden


@pytest.fixture(scope="module")
def host():
    from nvllm import host
    host.host_lib()
    return host


def test_allocator_replays_reference_trace(host):
    """tests/golden/allocator_trace.npz was recorded from the reference's
    PagedKVCache (src/kv_cache.cpp:23-55)."""
    g = load_golden("allocator_trace")
    a = host.BlockAllocator(int(g["num_blocks"]))
    pos = 0
    for i, (kind, arg) in enumerate(zip(g["op_kind"], g["op_arg"])):
        n = int(g["result_lens"][i])
        expect = g["result_ids"][pos:pos + n]
        if g["ok"][i]:
            pos += n
        if kind == 0:
            r = a.allocate_block()
            if g["ok"][i] and n:
                assert r == int(expect[0]), f"op {i}"
            else:
                assert r is None, f"op {i}"
        elif kind == 1:
            r = a.allocate_blocks(int(arg))
            if g["ok"][i]:
                assert r is not None and np.array_equal(r, expect), f"op {i}"
            else:
                assert r is None, f"op {i}"
        else:
            if n:
                assert a.free_blocks(expect) == 0
        assert a.num_free() == int(g["free_after"][i]), f"free count after op {i}"


def test_allocator_rejects_double_and_foreign_frees(host):
    a = host.BlockAllocator(8)
    ids = a.allocate_blocks(5)
    assert a.num_free() == 3
    assert a.allocate_blocks(4) is None  # all or nothing (tests/test_main.cpp:30-32)
    assert a.num_free() == 3
    assert a.free_blocks(ids) == 0
    assert a.num_free() == 8
    assert a.free_blocks([ids[0]]) == host.INVALID_BLOCK      # double free
    assert a.free_blocks([8]) == host.INVALID_BLOCK           # out of range
    one = a.allocate_block()
    assert a.free_blocks([one, one]) == host.INVALID_BLOCK    # duplicate in one call
    assert a.num_free() == 7                                  # rejected call changed nothing


def _tables_of(case):
    nb = (case.total_len + case.block_size - 1) // case.block_size
    return [case.block_tables[s, :nb[s]] for s in range(len(case.total_len))]


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c.name)
def test_packer_matches_golden(host, oracle, case):
    g = load_golden(case.name)
    mb = case.block_tables.shape[1] + 3
    m = host.pack_metadata(case.num_computed, case.total_len, _tables_of(case), case.block_size,
                           mb)
    assert np.array_equal(m["slot_mapping"], g["slot_mapping"])
    fl = oracle.flatten(case.num_computed, case.total_len)
    assert np.array_equal(m["cu_seqlens_q"], fl["cu_seqlens_q"])
    assert np.array_equal(m["context_lens"], fl["context_lens"])
    assert np.array_equal(m["last_token_idx"], fl["last_token_idx"])
    nb = case.block_tables.shape[1]
    assert np.array_equal(m["block_tables"][:, :nb], g["block_tables"])
    assert not m["block_tables"][:, nb:].any()
    assert m["max_query_len"] == int(case.q_lens.max())
    assert m["max_context_len"] == int(case.total_len.max())


def test_packer_random_batches(host, oracle):
    for seed in range(20):
        S = int(det_ints(seed, 1, 1, 1, 12)[0])
        total = det_ints(seed, 2, S, 1, 300)
        comp = np.minimum(total, det_ints(seed, 3, S, 0, 300))
        B = [1, 2, 3, 4, 8, 16, 32][seed % 7]
        case = make_case("r", seed, num_heads=1, head_dim=32, block_size=B, num_layers=1,
                         num_computed=comp, total_len=total)
        m = host.pack_metadata(case.num_computed, case.total_len, _tables_of(case), B,
                               case.block_tables.shape[1])
        fl = oracle.flatten(case.num_computed, case.total_len)
        sm = oracle.slot_mapping(fl["cu_seqlens_q"], fl["context_lens"], case.block_tables, B)
        assert np.array_equal(m["slot_mapping"], sm)
        assert np.array_equal(m["cu_seqlens_q"], fl["cu_seqlens_q"])
        assert np.array_equal(m["last_token_idx"], fl["last_token_idx"])


def test_packer_rejects_bad_batches(host):
    from nvllm import NvllmError
    with pytest.raises(NvllmError):  # table too short for 17 tokens at block size 16
        host.pack_metadata([0], [17], [[3]], 16, 4)
    with pytest.raises(NvllmError):  # more blocks than the table width
        host.pack_metadata([0], [40], [[1, 2, 3]], 16, 2)
    with pytest.raises(NvllmError):  # num_computed > total_len
        host.pack_metadata([5], [4], [[0]], 16, 4)
    m = host.pack_metadata([], [], [], 16, 4)  # empty batch
    assert m["cu_seqlens_q"].tolist() == [0]


def test_packer_padding_to_a_bucket(host, oracle):
    """A batch laid out as a bigger bucket: the real part is the unpadded
    packing unchanged, the extra sequences are empty and the extra rows have
    slot -1 (which the KV write skips)."""
    from nvllm import NvllmError
    for seed in range(10):
        S = int(det_ints(seed, 1, 1, 1, 9)[0])
        total = det_ints(seed, 2, S, 1, 200)
        comp = np.minimum(total, det_ints(seed, 3, S, 0, 200))
        B = [4, 8, 16][seed % 3]
        case = make_case("p", seed, num_heads=1, head_dim=32, block_size=B, num_layers=1,
                         num_computed=comp, total_len=total)
        W = case.block_tables.shape[1]
        plain = host.pack_metadata(case.num_computed, case.total_len, _tables_of(case), B, W)
        T = len(plain["slot_mapping"])
        pS, pT = S + 3, T + 5
        m = host.pack_metadata(case.num_computed, case.total_len, _tables_of(case), B, W,
                               pad_seqs=pS, pad_tokens=pT)
        assert np.array_equal(m["cu_seqlens_q"][:S + 1], plain["cu_seqlens_q"])
        assert (m["cu_seqlens_q"][S + 1:] == T).all()
        assert np.array_equal(m["context_lens"][:S], plain["context_lens"])
        assert (m["context_lens"][S:] == 0).all()
        assert np.array_equal(m["last_token_idx"][:S], plain["last_token_idx"])
        assert (m["last_token_idx"][S:] == 0).all()
        assert np.array_equal(m["slot_mapping"][:T], plain["slot_mapping"])
        assert (m["slot_mapping"][T:] == -1).all() and len(m["slot_mapping"]) == pT
        assert np.array_equal(m["block_tables"][:S], plain["block_tables"])
        assert (m["block_tables"][S:] == 0).all()
    with pytest.raises(NvllmError):  # a bucket smaller than the batch
        host.pack_metadata([0, 0], [3, 3], [[1], [2]], 16, 2, pad_seqs=1, pad_tokens=8)


def _reference_tokenize(text: str, vocab: int) -> list[int]:
    """The reference engine's tokenize_prompt (src/engine.cpp:40-64), restated:
    whitespace-separated words, each djb2-hashed into [1, vocab)."""
    out = []
    for word in text.replace("\t", " ").replace("\n", " ").replace("\r", " ").split(" "):
        if not word:
            continue
        h = 5381
        for b in word.encode():
            h = (h * 33 + b) & 0xFFFFFFFFFFFFFFFF
        out.append(h % (vocab - 1) + 1)
    return out or [1]


def test_prompt_tokenisation_follows_the_reference():
    from nvllm.host import tokenize_prompt
    cases = ["paged attention on blackwell", "", "   ", "a", "cpp26\tkernel\nstream\r\nx",
             "a-very-long-word-" * 40, "ünïcödé words"]
    for vocab in (2, 512, 32000):
        for text in cases:
            assert tokenize_prompt(text, vocab).tolist() == _reference_tokenize(text, vocab), text
    # djb2("a") = 5381 * 33 + 97
    assert tokenize_prompt("a", 512).tolist() == [(5381 * 33 + 97) % 511 + 1]
