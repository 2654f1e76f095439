"""Synthetic batches with the shapes of the paged-attention workloads.

* decode:  64 sequences, one query row each, contexts uniform in [512, 4096],
           32 heads x head_dim 128 (hidden 4096), block size 16, physical
           blocks from a seeded permutation of a 65536-block arena, Q/K/V and
           the cached KV ~ N(0, 1), softmax scale 1/sqrt(128);
* mixed:   8 fresh causal prefills of length U[512, 2048] + 120 decodes with
           contexts U[256, 8192], same geometry;
* longctx: 4 sequences with 32768-position contexts, same geometry;
* decode_small: the decode distribution with 16 sequences on a 4096-block
  arena (2 GiB K+V, ~1.2 GB read per call: still far beyond L2), the case for
  multi-pass profiler captures;
* mixed_small: the mixed distribution with 2 prefills and 8 decodes on a
  4096-block arena, the profiler case of the prefill kernels.

Context lengths and block tables come from numpy's PCG64 with the given seed;
tensor values from torch's CUDA generator. No public dataset is involved.

Sequence partitioning (one batch per GPU): rank r > 0 gets the same multiset of
context lengths as rank 0, in an order and with block tables drawn from a
generator seeded with (seed, r), so every GPU moves the same bytes and the
curve over GPU counts measures the system rather than unequal batches.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

WORKLOADS = {
    "decode": dict(num_heads=32, head_dim=128, block_size=16, num_blocks=65536),
    "mixed": dict(num_heads=32, head_dim=128, block_size=16, num_blocks=65536),
    "longctx": dict(num_heads=32, head_dim=128, block_size=16, num_blocks=8192 + 64),
    "decode_small": dict(num_heads=32, head_dim=128, block_size=16, num_blocks=4096),
    "mixed_small": dict(num_heads=32, head_dim=128, block_size=16, num_blocks=4096),
}


@dataclass
class BatchSpec:
    name: str
    num_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    ctx_lens: np.ndarray     # [S] KV positions after this step's write
    q_lens: np.ndarray       # [S] query rows this step
    block_tables: np.ndarray  # [S, max_blocks] int32

    @property
    def hidden(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def num_seqs(self) -> int:
        return len(self.ctx_lens)

    @property
    def cu_seqlens_q(self) -> np.ndarray:
        return np.concatenate([[0], np.cumsum(self.q_lens)]).astype(np.int32)

    @property
    def n_tokens(self) -> int:
        return int(self.q_lens.sum())

    def slot_mapping(self) -> np.ndarray:
        """block_table[pos / B] * B + pos % B for every new token
        (src/model.cpp:192-194)."""
        out = np.empty(self.n_tokens, np.int32)
        cu = self.cu_seqlens_q
        B = self.block_size
        for s in range(self.num_seqs):
            pos = np.arange(self.ctx_lens[s] - self.q_lens[s], self.ctx_lens[s])
            out[cu[s]:cu[s + 1]] = self.block_tables[s, pos // B] * B + pos % B
        return out

    def kv_bytes(self) -> int:
        """K+V bytes the attention must read: every cached position of every
        head once."""
        return int(self.ctx_lens.astype(np.int64).sum()) * self.hidden * 4 * 2

    def decode_algorithmic_bytes(self) -> int:
        """HBM bytes one attention call must move: K and V of every visible
        position, Q in and O out, block-table entries and per-sequence
        metadata."""
        nb = (self.ctx_lens + self.block_size - 1) // self.block_size
        return (self.kv_bytes() + self.n_tokens * self.hidden * 4 * 2 + int(nb.sum()) * 4 +
                self.num_seqs * 8 + 4)

    def subset(self, seqs) -> "BatchSpec":
        """The batch restricted to the sequences ``seqs`` (same arena, same
        tables)."""
        seqs = np.asarray(seqs, np.int64)
        nb = (self.ctx_lens[seqs] + self.block_size - 1) // self.block_size
        width = max(int(nb.max()) if len(nb) else 1, 1)
        return BatchSpec(name=self.name, num_heads=self.num_heads, head_dim=self.head_dim,
                         block_size=self.block_size, num_blocks=self.num_blocks,
                         ctx_lens=self.ctx_lens[seqs].copy(), q_lens=self.q_lens[seqs].copy(),
                         block_tables=np.ascontiguousarray(self.block_tables[seqs, :width]))

    def prefill_flops(self) -> int:
        """QK^T + PV FLOPs of the multi-row sequences (causal)."""
        f = 0
        for c, q in zip(self.ctx_lens.tolist(), self.q_lens.tolist()):
            if q > 1:
                first = c - q
                keys = sum(first + i + 1 for i in range(q))
                f += 4 * self.hidden * keys
        return f


def _tables(rng, ctx, block_size, num_blocks):
    nbs = (ctx + block_size - 1) // block_size
    assert nbs.sum() <= num_blocks
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((len(ctx), int(nbs.max())), np.int32)
    off = 0
    for s, nb in enumerate(nbs.tolist()):
        bt[s, :nb] = perm[off:off + nb]
        off += nb
    return bt


def make_batch(name: str = "decode", seed: int = 0, rank: int = 0) -> BatchSpec:
    geo = WORKLOADS[name]
    rng = np.random.Generator(np.random.PCG64(seed))
    if name == "decode":
        ctx = rng.integers(512, 4096, size=64, endpoint=True).astype(np.int32)
        ql = np.ones(64, np.int32)
    elif name == "mixed":
        pre = rng.integers(512, 2048, size=8, endpoint=True).astype(np.int32)
        dec = rng.integers(256, 8192, size=120, endpoint=True).astype(np.int32)
        ctx = np.concatenate([pre, dec]).astype(np.int32)
        ql = np.concatenate([pre, np.ones(120, np.int32)]).astype(np.int32)
    elif name == "mixed_small":
        pre = rng.integers(512, 2048, size=2, endpoint=True).astype(np.int32)
        dec = rng.integers(256, 8192, size=8, endpoint=True).astype(np.int32)
        ctx = np.concatenate([pre, dec]).astype(np.int32)
        ql = np.concatenate([pre, np.ones(8, np.int32)]).astype(np.int32)
    elif name == "decode_small":
        ctx = rng.integers(512, 4096, size=16, endpoint=True).astype(np.int32)
        ql = np.ones(16, np.int32)
    elif name == "longctx":
        ctx = np.full(4, 32768, np.int32)
        ql = np.ones(4, np.int32)
    else:
        raise KeyError(name)
    if rank:
        # same lengths, another order within the prefill and the decode group,
        # other physical blocks
        rng = np.random.Generator(np.random.PCG64([seed, rank]))
        pre = np.flatnonzero(ql > 1)
        dec = np.flatnonzero(ql == 1)
        order = np.concatenate([rng.permutation(pre), rng.permutation(dec)])
        ctx, ql = ctx[order], ql[order]
    bt = _tables(rng, ctx, geo["block_size"], geo["num_blocks"])
    return BatchSpec(name=name, num_heads=geo["num_heads"], head_dim=geo["head_dim"],
                     block_size=geo["block_size"], num_blocks=geo["num_blocks"], ctx_lens=ctx,
                     q_lens=ql, block_tables=bt)
