"""Parity of the CUDA path (through the C ABI) with the reference.

* golden fixtures: outputs of the reference's own forward_batch (max-abs
  TOL_FP32) and arena contents (bit-exact against the oracle's write_kv);
* seeded cases at the decode / mixed / long-context shapes against the C
  oracle on the same inputs (TOL_FP32);
* size-independent properties at the full decode-benchmark size (65536-block
  arena): bit-exact invariance under physical block relocation, a sampled
  oracle check, finiteness;
* edge cases and error reporting.
"""
import math

import numpy as np
import pytest

from helpers import (TOL_FP32, TOL_TF32, device_run, golden_case, golden_names, layout_of, load_golden,
                     oracle_run)

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names())
def test_golden_fixture(nv, oracle, name):
    case = golden_case(name)
    g = load_golden(name)
    ka, va, out, status = device_run(nv, oracle, case)
    assert status == nv.OK, nv.status_string(status)
    err = np.abs(out - g["attn_out"]).max()
    assert err <= TOL_FP32, f"{name}: kernel vs reference max-abs {err}"
    oka, ova, oout, _ = oracle_run(oracle, case)
    assert np.array_equal(ka, oka), "K arena must be bit-exact"
    assert np.array_equal(va, ova), "V arena must be bit-exact"
    assert np.abs(out - oout).max() <= TOL_FP32


# ---------------------------------------------------------------------------
# seeded device-generated batches


def _torch():
    import torch
    return torch


def build_batch(nv, *, seed, num_blocks, block_size, num_heads, head_dim, ctx_lens, q_lens,
                num_layers=1, layer=0, arena_fill=True, block_tables=None):
    """Device batch: arena filled with N(0,1), block tables from a seeded
    permutation (or the given ``block_tables``), the new tokens' K/V written by
    nvllm_reshape_and_cache, Q N(0,1). Returns a dict of device tensors and host
    metadata."""
    torch = _torch()
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    lay = nv.KVLayout(num_blocks, num_layers, block_size, num_heads, head_dim)
    D = num_heads * head_dim
    ka = torch.empty(lay.arena_shape(), dtype=torch.float32, device=dev)
    va = torch.empty_like(ka)
    if arena_fill:
        ka.normal_(generator=gen)
        va.normal_(generator=gen)
    else:
        ka.zero_()
        va.zero_()
    ctx_lens = np.asarray(ctx_lens, np.int32)
    q_lens = np.asarray(q_lens, np.int32)
    S = len(ctx_lens)
    nbs = (ctx_lens + block_size - 1) // block_size
    max_blocks = int(nbs.max())
    if block_tables is None:
        hg = torch.Generator()
        hg.manual_seed(seed)
        perm = torch.randperm(num_blocks, generator=hg).numpy().astype(np.int32)
        assert nbs.sum() <= num_blocks
        bt = np.zeros((S, max_blocks), np.int32)
        off = 0
        for s in range(S):
            bt[s, :nbs[s]] = perm[off:off + nbs[s]]
            off += nbs[s]
    else:
        bt = np.ascontiguousarray(block_tables, np.int32)
        assert bt.shape[0] == S and bt.shape[1] >= max_blocks
    cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    n = int(cu[-1])
    slots = np.zeros(n, np.int32)
    for s in range(S):
        for i in range(q_lens[s]):
            pos = ctx_lens[s] - q_lens[s] + i
            slots[cu[s] + i] = bt[s, pos // block_size] * block_size + pos % block_size
    q = torch.randn((n, D), generator=gen, device=dev)
    k = torch.randn((n, D), generator=gen, device=dev)
    v = torch.randn((n, D), generator=gen, device=dev)
    d = dict(lay=lay, ka=ka, va=va, bt=bt, cu=cu, ctx=ctx_lens, slots=slots, q=q, k=k, v=v,
             layer=layer, max_q=int(q_lens.max()), max_ctx=int(ctx_lens.max()))
    d["bt_d"] = torch.from_numpy(bt).to(dev)
    d["cu_d"] = torch.from_numpy(cu).to(dev)
    d["ctx_d"] = torch.from_numpy(ctx_lens).to(dev)
    d["slots_d"] = torch.from_numpy(slots).to(dev)
    nv.reshape_and_cache(k, v, ka, va, d["slots_d"], layer, lay)
    return d


def run_attention(nv, b, precision=0, workspace=None):
    torch = _torch()
    out = torch.full_like(b["q"], float("nan"))
    nv.paged_attention(out, b["q"], b["ka"], b["va"], b["bt_d"], b["cu_d"], b["ctx_d"], b["max_q"],
                       b["max_ctx"], b["layer"], b["lay"], precision=precision,
                       workspace=workspace)
    torch.cuda.synchronize()
    return out


def oracle_check(nv, oracle, b, out, seqs, tol=TOL_FP32, more=(), host_budget=2 << 30):
    """Compares the output rows of the chosen sequences with the oracle.

    The sequences go in groups whose blocks fit ``host_budget`` bytes of host
    memory (K + V); each group's blocks are copied into a compact host arena and
    the oracle attends them once. ``out`` is checked within ``tol`` and every
    further ``(output, tol)`` pair of ``more`` (the same batch computed another
    way) against the same oracle rows. Returns the largest error of ``out``."""
    torch = _torch()
    lay = b["lay"]
    nbs = (b["ctx"] + lay.block_size - 1) // lay.block_size
    row_bytes = 2 * lay.num_layers * lay.block_size * lay.num_heads * lay.head_dim * 4
    groups, cur, cur_blocks = [], [], 0
    for s in seqs:
        if cur and (cur_blocks + int(nbs[s])) * row_bytes > host_budget:
            groups.append(cur)
            cur, cur_blocks = [], 0
        cur.append(s)
        cur_blocks += int(nbs[s])
    if cur:
        groups.append(cur)
    worst = 0.0
    for g in groups:
        ref, q_rows = _oracle_rows(oracle, b, g)
        for o, t in ((out, tol), *more):
            got = o[torch.as_tensor(q_rows, device=o.device)].cpu().numpy()
            err = float(np.abs(got - ref).max()) if len(q_rows) else 0.0
            assert err <= t, f"sequences {g[0]}..{g[-1]}: max-abs {err} > {t}"
            if o is out:
                worst = max(worst, err)
    return worst


def _oracle_rows(oracle, b, seqs):
    """The oracle's output rows for ``seqs`` (and their row indices in the
    batch), from a compact host copy of the blocks those sequences use."""
    from oracle.oracle import KVLayout
    torch = _torch()
    lay = b["lay"]
    bt = b["bt"]
    nbs = (b["ctx"] + lay.block_size - 1) // lay.block_size
    used = []
    for s in seqs:
        used.extend(bt[s, :nbs[s]].tolist())
    used = np.array(sorted(set(used)), np.int64)
    remap = {int(x): i for i, x in enumerate(used)}
    idx = torch.from_numpy(used).to(b["ka"].device)
    ka = b["ka"].index_select(0, idx).cpu().numpy()
    va = b["va"].index_select(0, idx).cpu().numpy()
    S = len(seqs)
    bt_c = np.zeros((S, bt.shape[1]), np.int32)
    q_rows, cu = [], [0]
    for j, s in enumerate(seqs):
        bt_c[j, :nbs[s]] = [remap[int(x)] for x in bt[s, :nbs[s]]]
        q_rows.extend(range(b["cu"][s], b["cu"][s + 1]))
        cu.append(len(q_rows))
    q = b["q"][torch.as_tensor(q_rows, device=b["q"].device)].cpu().numpy()
    olay = KVLayout(len(used), lay.num_layers, lay.block_size, lay.num_heads, lay.head_dim)
    ref = oracle.paged_attention(q, ka, va, bt_c, np.array(cu, np.int32),
                                 b["ctx"][list(seqs)].astype(np.int32), b["layer"],
                                 1.0 / math.sqrt(lay.head_dim), olay)
    return ref, q_rows


def test_decode_shape_vs_oracle(nv, oracle):
    """32 heads x hd 128, block 16, contexts U[512, 4096] (decode microbench
    shape, 16 sequences)."""
    rng = np.random.default_rng(1)
    ctx = rng.integers(512, 4097, 16).astype(np.int32)
    b = build_batch(nv, seed=11, num_blocks=8192, block_size=16, num_heads=32, head_dim=128,
                    ctx_lens=ctx, q_lens=np.ones(16, np.int32))
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, list(range(16)))


def test_mixed_shape_vs_oracle(nv, oracle):
    """Flattened prefill + decode batch shaped like the 4096-hidden layer:
    2 fresh causal prefills, one chunked continuation, 20 decodes."""
    rng = np.random.default_rng(2)
    dec = rng.integers(256, 3001, 20).astype(np.int32)
    ctx = np.concatenate([[700, 333, 900], dec]).astype(np.int32)
    ql = np.concatenate([[700, 333, 150], np.ones(20)]).astype(np.int32)
    b = build_batch(nv, seed=12, num_blocks=8192, block_size=16, num_heads=32, head_dim=128,
                    ctx_lens=ctx, q_lens=ql)
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, list(range(len(ctx))))


@pytest.mark.parametrize("head_dim,block_size", [(32, 16), (64, 8), (256, 16), (128, 1),
                                                 (128, 32), (64, 3)])
def test_head_dims_and_block_sizes(nv, oracle, head_dim, block_size):
    rng = np.random.default_rng(head_dim + block_size)
    dec = rng.integers(1, 1500, 9).astype(np.int32)
    ctx = np.concatenate([[130, 64, 77], dec]).astype(np.int32)
    ql = np.concatenate([[130, 2, 65], np.ones(9)]).astype(np.int32)
    H = 4096 // head_dim // 4
    nb = int(((ctx + block_size - 1) // block_size).sum()) + 5
    b = build_batch(nv, seed=13, num_blocks=nb, block_size=block_size, num_heads=H,
                    head_dim=head_dim, ctx_lens=ctx, q_lens=ql, num_layers=2, layer=1)
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, list(range(len(ctx))))


def test_split_boundaries(nv, oracle):
    """Contexts at and around the decode split size and chunk size."""
    P = 256  # positions per decode item at hd 128
    ctx = np.array([1, 15, 16, 17, P - 1, P, P + 1, 2 * P, 2 * P + 1, 16 * P, 16 * P + 3],
                   np.int32)
    b = build_batch(nv, seed=14, num_blocks=4096, block_size=16, num_heads=8, head_dim=128,
                    ctx_lens=ctx, q_lens=np.ones(len(ctx), np.int32))
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, list(range(len(ctx))))


def test_long_context_decode(nv, oracle):
    """Long-context shape: 4 sequences x 32768 positions, 32 heads x hd 128."""
    ctx = np.full(4, 32768, np.int32)
    b = build_batch(nv, seed=15, num_blocks=8192 + 16, block_size=16, num_heads=32, head_dim=128,
                    ctx_lens=ctx, q_lens=np.ones(4, np.int32))
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, [0, 1, 2, 3])


def test_decode_benchmark_full_size(nv, oracle):
    """The decode benchmark's batch: 64 sequences, contexts U[512, 4096],
    block tables from the seeded permutation of the 65536-block arena (34 GB
    K+V) that the benchmark uses; every sequence against the oracle,
    finiteness, and bit-exact invariance of the output under relocation of
    every physical block."""
    from nvllm.workload import make_batch
    torch = _torch()
    spec = make_batch("decode", seed=0)
    b = build_batch(nv, seed=16, num_blocks=65536, block_size=16, num_heads=32, head_dim=128,
                    ctx_lens=spec.ctx_lens, q_lens=spec.q_lens, block_tables=spec.block_tables)
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    assert torch.isfinite(out).all()
    oracle_check(nv, oracle, b, out, list(range(64)))
    # relocate: physical block j -> perm[j]; tables rewritten accordingly
    g = torch.Generator()
    g.manual_seed(99)
    perm = torch.randperm(65536, generator=g).to(b["ka"].device)
    ka2 = torch.empty_like(b["ka"])
    ka2[perm] = b["ka"]
    b["ka"] = ka2
    va2 = torch.empty_like(b["va"])
    va2[perm] = b["va"]
    b["va"] = va2
    del ka2, va2
    b["bt_d"] = perm[b["bt_d"].long()].to(torch.int32)
    out2 = run_attention(nv, b)
    assert torch.equal(out, out2), "output must not depend on physical placement"


def test_mixed_benchmark_full_size(nv, oracle):
    """The mixed super-batch exactly as benchmarked: 8 fresh causal prefills of
    U[512, 2048] rows + 120 decodes with contexts U[256, 8192], 32 heads x hd 128,
    block size 16, block tables from the seeded permutation of the 65536-block
    arena. All 128 sequences (8376 query rows) against the oracle, with fp32
    prefill tiles (TOL_FP32) and with tensor-core tiles (TOL_TF32)."""
    from nvllm.workload import make_batch
    torch = _torch()
    spec = make_batch("mixed", seed=0)
    assert spec.num_seqs == 128 and int((spec.q_lens > 1).sum()) == 8
    b = build_batch(nv, seed=30, num_blocks=65536, block_size=16, num_heads=32, head_dim=128,
                    ctx_lens=spec.ctx_lens, q_lens=spec.q_lens, block_tables=spec.block_tables)
    ws = nv.alloc_workspace(spec.num_seqs, b["max_q"], b["max_ctx"], b["lay"],
                            device=b["q"].device)
    out = run_attention(nv, b, workspace=ws)
    assert nv.get_last_error() == nv.OK
    out_tc = run_attention(nv, b, precision=nv.PRECISION_TF32, workspace=ws)
    assert nv.get_last_error() == nv.OK
    assert torch.isfinite(out).all() and torch.isfinite(out_tc).all()
    err = oracle_check(nv, oracle, b, out, list(range(spec.num_seqs)),
                       more=[(out_tc, TOL_TF32)])
    assert err <= TOL_FP32


def test_longctx_benchmark_full_size(nv, oracle):
    """The long-context batch as benchmarked (4 x 32768 positions, block tables
    from the benchmark's seeded permutation): all 4 sequences against the
    oracle, and every head-group slice of it (heads split over 2, 4 and 8
    ranks, each slice attended on its own arena slice, as a rank of the head
    split does) bit-identical to the matching columns of the whole: a head's
    arithmetic does not depend on how many heads share the call."""
    from nvllm.workload import make_batch
    torch = _torch()
    spec = make_batch("longctx", seed=0)
    b = build_batch(nv, seed=31, num_blocks=spec.num_blocks, block_size=16, num_heads=32,
                    head_dim=128, ctx_lens=spec.ctx_lens, q_lens=spec.q_lens,
                    block_tables=spec.block_tables)
    out = run_attention(nv, b)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, [0, 1, 2, 3])
    hd = 128
    for n in (2, 4, 8):
        hl = 32 // n
        for r in (0, n - 1):
            cols = slice(r * hl * hd, (r + 1) * hl * hd)
            lay = nv.KVLayout(spec.num_blocks, 1, 16, hl, hd)
            ka = b["ka"][..., cols].contiguous()
            va = b["va"][..., cols].contiguous()
            q = b["q"][:, cols].contiguous()
            part = torch.full_like(q, float("nan"))
            nv.paged_attention(part, q, ka, va, b["bt_d"], b["cu_d"], b["ctx_d"], 1,
                               b["max_ctx"], 0, lay)
            torch.cuda.synchronize()
            assert nv.get_last_error() == nv.OK
            assert torch.equal(part, out[:, cols]), f"heads split {n} ways, rank {r}"
            del ka, va


def test_constant_values_give_constant_output(nv):
    """Softmax weights sum to one: V rows all equal c => output == c."""
    torch = _torch()
    ctx = np.array([1, 100, 1000, 5000], np.int32)
    b = build_batch(nv, seed=17, num_blocks=1024, block_size=16, num_heads=4, head_dim=128,
                    ctx_lens=ctx, q_lens=np.array([1, 1, 1, 1], np.int32))
    b["va"].fill_(0.375)
    out = run_attention(nv, b)
    assert torch.allclose(out, torch.full_like(out, 0.375), atol=1e-6, rtol=0)


def test_reshape_and_cache_negative_slot_and_bit_exact(nv):
    torch = _torch()
    dev = torch.device("cuda:0")
    lay = nv.KVLayout(8, 2, 4, 2, 32)
    ka = torch.zeros(lay.arena_shape(), device=dev)
    va = torch.zeros_like(ka)
    k = torch.randn(3, 64, device=dev)
    v = torch.randn(3, 64, device=dev)
    slots = torch.tensor([5, -1, 31], dtype=torch.int32, device=dev)
    nv.reshape_and_cache(k, v, ka, va, slots, 1, lay)
    assert nv.get_last_error() == nv.OK
    exp_k = torch.zeros_like(ka)
    exp_k[1, 1, 1] = k[0]
    exp_k[7, 1, 3] = k[2]
    assert torch.equal(ka, exp_k)
    assert torch.equal(va[1, 1, 1], v[0]) and torch.equal(va[7, 1, 3], v[2])


def test_out_of_range_block_is_reported(nv):
    torch = _torch()
    b = build_batch(nv, seed=18, num_blocks=64, block_size=16, num_heads=2, head_dim=64,
                    ctx_lens=[40, 20], q_lens=[1, 1], arena_fill=False)
    bt = b["bt_d"].clone()
    bt[0, 1] = 64  # one past the arena
    b["bt_d"] = bt
    run_attention(nv, b)
    assert nv.get_last_error() == nv.ERR_BOUNDS
    assert nv.get_last_error() == nv.OK  # cleared
    lay = b["lay"]
    bad = torch.tensor([64 * 16], dtype=torch.int32, device="cuda")
    nv.reshape_and_cache(b["k"][:1], b["v"][:1], b["ka"], b["va"], bad, 0, lay)
    assert nv.get_last_error() == nv.ERR_BOUNDS


def test_inconsistent_metadata_is_reported(nv):
    b = build_batch(nv, seed=19, num_blocks=64, block_size=16, num_heads=2, head_dim=64,
                    ctx_lens=[40, 20], q_lens=[1, 1], arena_fill=False)
    b["max_ctx"] = 30  # sequence 0 has 40 > 30
    run_attention(nv, b)
    assert nv.get_last_error() == nv.ERR_INVALID


def test_argument_errors(nv):
    torch = _torch()
    b = build_batch(nv, seed=20, num_blocks=64, block_size=16, num_heads=2, head_dim=64,
                    ctx_lens=[40, 20], q_lens=[1, 1], arena_fill=False)
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    st = nv.paged_attention(torch.empty_like(b["q"]), b["q"], b["ka"], b["va"], b["bt_d"],
                            b["cu_d"], b["ctx_d"], 1, 40, 0, b["lay"], workspace=small,
                            check=False)
    assert st == nv.ERR_WORKSPACE
    bad = nv.KVLayout(64, 1, 16, 2, 48)
    assert nv.workspace_size(2, 1, 40, bad) == 0
    st = nv.reshape_and_cache(b["k"], b["v"], b["ka"], b["va"], b["slots_d"], 0, bad, check=False)
    assert st == nv.ERR_UNSUPPORTED
    st = nv.reshape_and_cache(b["k"], b["v"], b["ka"], b["va"], b["slots_d"], 5, b["lay"],
                              check=False)
    assert st == nv.ERR_INVALID
    # max_context_len beyond the table capacity
    st = nv.paged_attention(torch.empty_like(b["q"]), b["q"], b["ka"], b["va"], b["bt_d"],
                            b["cu_d"], b["ctx_d"], 1, 10_000, 0, b["lay"], check=False)
    assert st == nv.ERR_INVALID


def test_empty_batch_is_noop(nv):
    torch = _torch()
    lay = nv.KVLayout(4, 1, 16, 2, 64)
    z = torch.zeros(0, 128, device="cuda")
    ka = torch.zeros(lay.arena_shape(), device="cuda")
    i0 = torch.zeros(0, dtype=torch.int32, device="cuda")
    assert nv.reshape_and_cache(z, z, ka, ka.clone(), i0, 0, lay) == nv.OK
    cu = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.empty(256, dtype=torch.uint8, device="cuda")
    st = nv.paged_attention(z, z, ka, ka, torch.zeros(0, 1, dtype=torch.int32, device="cuda"), cu,
                            i0, 1, 1, 0, lay, workspace=ws)
    assert st == nv.OK


# ---------------------------------------------------------------------------
# TF32 tensor-core prefill (tcgen05): tolerance 1e-3


@pytest.mark.parametrize("name", ["mixed_h32_hd128_b16", "decode_h32_hd128_b16",
                                  "mixed_h4_hd32_b4"])
def test_golden_fixture_tf32(nv, oracle, name):
    case = golden_case(name)
    g = load_golden(name)
    _, _, out, status = device_run(nv, oracle, case, precision=nv.PRECISION_TF32)
    assert status == nv.OK, nv.status_string(status)
    err = np.abs(out - g["attn_out"]).max()
    assert err <= TOL_TF32, f"{name}: tf32 kernel vs reference max-abs {err}"


def test_tf32_prefill_mixed_shape_vs_oracle(nv, oracle):
    """Fresh causal prefills (row counts around the 128-row tile and the
    64-key tile), a chunked continuation and decodes, TF32 prefill tiles."""
    rng = np.random.default_rng(21)
    dec = rng.integers(256, 3001, 12).astype(np.int32)
    ctx = np.concatenate([[700, 128, 129, 64, 65, 2, 900], dec]).astype(np.int32)
    ql = np.concatenate([[700, 128, 129, 64, 65, 2, 150], np.ones(12)]).astype(np.int32)
    b = build_batch(nv, seed=22, num_blocks=4096, block_size=16, num_heads=32, head_dim=128,
                    ctx_lens=ctx, q_lens=ql)
    out = run_attention(nv, b, precision=nv.PRECISION_TF32)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, list(range(len(ctx))), tol=TOL_TF32)


def test_tf32_prefill_stale_nonfinite_rows_do_not_leak(nv, oracle):
    """Arena rows past a sequence's end inside its last block hold NaN: the
    tensor-core tile loads whole blocks, so those rows must be neutralised."""
    torch = _torch()
    ctx = np.array([37, 200, 90], np.int32)
    ql = np.array([37, 200, 20], np.int32)
    b = build_batch(nv, seed=23, num_blocks=256, block_size=16, num_heads=4, head_dim=128,
                    ctx_lens=ctx, q_lens=ql)
    # poison every row past each sequence's last position in its last block
    for s in range(len(ctx)):
        last = int(b["bt"][s, (ctx[s] - 1) // 16])
        for slot in range(ctx[s] % 16 or 16, 16):
            b["ka"][last, 0, slot] = float("nan")
            b["va"][last, 0, slot] = float("nan")
    for precision, tol in ((nv.PRECISION_TF32, TOL_TF32), (nv.PRECISION_FP32, TOL_FP32)):
        out = run_attention(nv, b, precision=precision)
        assert nv.get_last_error() == nv.OK
        assert torch.isfinite(out).all()
        oracle_check(nv, oracle, b, out, [0, 1, 2], tol=tol)


def test_tf32_other_geometries_use_fp32_prefill(nv, oracle):
    b = build_batch(nv, seed=24, num_blocks=512, block_size=8, num_heads=8, head_dim=64,
                    ctx_lens=[300, 40, 700], q_lens=[300, 1, 33])
    out = run_attention(nv, b, precision=nv.PRECISION_TF32)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, [0, 1, 2], tol=TOL_FP32)


def test_tf32_prefill_tile_boundaries(nv, oracle):
    """Prefills whose row counts straddle the tensor-core kernel's 128-row
    query tiles and 64-key tiles (and multiples of those), fresh and chunked
    (rows starting mid-context), with decodes beside them; every row against
    the oracle at the TF32 tolerance."""
    ctx = np.array([255, 256, 257, 511, 513, 100, 640, 300, 1000, 77, 3000, 191, 193], np.int32)
    ql = np.array([255, 256, 257, 511, 513, 100, 260, 44, 129, 1, 1, 63, 129], np.int32)
    b = build_batch(nv, seed=42, num_blocks=2048, block_size=16, num_heads=8, head_dim=128,
                    ctx_lens=ctx, q_lens=ql)
    out = run_attention(nv, b, precision=nv.PRECISION_TF32)
    assert nv.get_last_error() == nv.OK
    oracle_check(nv, oracle, b, out, list(range(len(ctx))), tol=TOL_TF32)
