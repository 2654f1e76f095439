"""Deterministic batches for the paged-KV write + attention tests.

Inputs come from a counter-based generator (splitmix64 -> Box-Muller in
float64 -> float32) so that a case is fully defined by its seed and shape,
independent of numpy's Generator streams. The golden fixtures store only the
case description, input checksums and the reference outputs.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix64(x: np.ndarray) -> np.ndarray:
    x = (x + np.uint64(0x9E3779B97F4A7C15)) & _M64
    z = x
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & _M64
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & _M64
    return z ^ (z >> np.uint64(31))


def det_uniform(seed: int, stream: int, n: int) -> np.ndarray:
    """n float64 uniforms in (0, 1)."""
    base = np.uint64((seed * 0x100000001B3 + stream * 0xC2B2AE3D27D4EB4F) & 0xFFFFFFFFFFFFFFFF)
    with np.errstate(over="ignore"):
        ctr = np.arange(n, dtype=np.uint64) + base
        bits = _splitmix64(ctr)
    return ((bits >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def det_normal(seed: int, stream: int, n: int) -> np.ndarray:
    """n standard normals as float32 (Box-Muller on two uniform streams)."""
    m = (n + 1) // 2
    u1 = det_uniform(seed, 2 * stream, m)
    u2 = det_uniform(seed, 2 * stream + 1, m)
    r = np.sqrt(-2.0 * np.log(u1))
    z = np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)])[:n]
    return z.astype(np.float32)


def det_permutation(seed: int, stream: int, n: int) -> np.ndarray:
    return np.argsort(det_uniform(seed, stream, n), kind="stable").astype(np.int32)


def det_ints(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    """n integers uniform in [lo, hi]."""
    u = det_uniform(seed, stream, n)
    return (lo + np.floor(u * (hi - lo + 1))).astype(np.int32)


@dataclass
class Case:
    """A batch for one step of the path. Sequence s has total_len[s] tokens,
    the first num_computed[s] already cached (their K/V in hist_k/hist_v,
    [L, sum num_computed, D], sequence-major); the rest are this step's new
    tokens with projections q/k/v [L, n_tok, D] in flatten order."""

    name: str
    seed: int
    num_blocks: int
    num_layers: int
    block_size: int
    num_heads: int
    head_dim: int
    num_computed: np.ndarray
    total_len: np.ndarray
    block_tables: np.ndarray
    hist_k: np.ndarray = field(repr=False)
    hist_v: np.ndarray = field(repr=False)
    q: np.ndarray = field(repr=False)
    k: np.ndarray = field(repr=False)
    v: np.ndarray = field(repr=False)

    @property
    def hidden(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def q_lens(self) -> np.ndarray:
        return (self.total_len - self.num_computed).astype(np.int32)

    @property
    def n_tokens(self) -> int:
        return int(self.q_lens.sum())

    @property
    def scale(self) -> float:
        return float(np.float32(1.0) / np.sqrt(np.float32(self.head_dim)))

    def checksums(self) -> dict:
        out = {}
        for nm in ("hist_k", "hist_v", "q", "k", "v"):
            a = getattr(self, nm)
            out[nm] = float(np.float64(a.astype(np.float64).sum()))
        return out


def make_case(name: str, seed: int, *, num_heads: int, head_dim: int, block_size: int,
              num_layers: int, num_computed, total_len, num_blocks: int | None = None,
              spare_blocks: int = 7) -> Case:
    num_computed = np.asarray(num_computed, np.int32)
    total_len = np.asarray(total_len, np.int32)
    assert np.all(total_len >= 1) and np.all(num_computed <= total_len)
    nb_per_seq = (total_len + block_size - 1) // block_size
    need = int(nb_per_seq.sum())
    if num_blocks is None:
        num_blocks = need + spare_blocks
    assert num_blocks >= need
    perm = det_permutation(seed, 1, num_blocks)
    max_blocks = max(int(nb_per_seq.max()), 1)
    bt = np.zeros((len(total_len), max_blocks), np.int32)
    off = 0
    for s, nb in enumerate(nb_per_seq):
        bt[s, :nb] = perm[off:off + nb]
        off += int(nb)
    d = num_heads * head_dim
    n_hist = int(num_computed.sum())
    n_new = int((total_len - num_computed).sum())
    L = num_layers

    def normal(stream, rows):
        return det_normal(seed, stream, L * rows * d).reshape(L, rows, d)

    return Case(name=name, seed=seed, num_blocks=num_blocks, num_layers=L,
                block_size=block_size, num_heads=num_heads, head_dim=head_dim,
                num_computed=num_computed, total_len=total_len, block_tables=bt,
                hist_k=normal(10, n_hist), hist_v=normal(11, n_hist),
                q=normal(12, n_new), k=normal(13, n_new), v=normal(14, n_new))


def golden_cases() -> list[Case]:
    """The cases whose reference outputs are committed under tests/golden/."""
    cases = []
    # Reference default model dims (include/nano_vllm/model.hpp:14-21): H 4,
    # hd 32, 2 layers; block size 16 (kv_cache.hpp:20). Pure decode, ragged
    # contexts including a single-token context and exact block multiples.
    ctx = np.array([1, 2, 15, 16, 17, 31, 32, 33, 64, 80], np.int32)
    cases.append(make_case("decode_h4_hd32_b16", 101, num_heads=4, head_dim=32, block_size=16,
                           num_layers=2, num_computed=ctx - 1, total_len=ctx))
    # Mixed prefill + decode + chunked continuation, block size 4 (the
    # reference's allocation test uses block size 4, tests/test_main.cpp:16-22).
    cases.append(make_case("mixed_h4_hd32_b4", 102, num_heads=4, head_dim=32, block_size=4,
                           num_layers=2, num_computed=[0, 0, 7, 12, 3, 0],
                           total_len=[5, 1, 8, 29, 11, 13]))
    # Block size 2 and 8 (tests/test_main.cpp:39-75, :77-124 configs).
    cases.append(make_case("mixed_h2_hd64_b2", 103, num_heads=2, head_dim=64, block_size=2,
                           num_layers=1, num_computed=[0, 4, 9], total_len=[4, 5, 12]))
    cases.append(make_case("mixed_h4_hd32_b8", 104, num_heads=4, head_dim=32, block_size=8,
                           num_layers=2, num_computed=[0, 17, 40, 0], total_len=[19, 18, 41, 2]))
    # Attention shaped like the 4096-hidden, 32-head, hd-128 layer of the
    # decode and mixed-batch workloads, at sizes the fixture can hold.
    cases.append(make_case("decode_h32_hd128_b16", 105, num_heads=32, head_dim=128,
                           block_size=16, num_layers=1,
                           num_computed=[0, 15, 16, 47, 200, 511],
                           total_len=[1, 16, 17, 48, 201, 512]))
    cases.append(make_case("mixed_h32_hd128_b16", 106, num_heads=32, head_dim=128,
                           block_size=16, num_layers=1, num_computed=[0, 100, 0, 33],
                           total_len=[19, 101, 3, 34]))
    # Head dims 64 and 256.
    cases.append(make_case("mixed_h8_hd64_b16", 107, num_heads=8, head_dim=64, block_size=16,
                           num_layers=1, num_computed=[0, 60, 99], total_len=[23, 61, 100]))
    cases.append(make_case("mixed_h2_hd256_b16", 108, num_heads=2, head_dim=256, block_size=16,
                           num_layers=1, num_computed=[0, 70], total_len=[19, 71]))
    return cases


def bimodal_workload(num_requests: int, vocab: int):
    """The reference benchmark's request set (src/benchmark.cpp:46-67):
    request i has a prompt of 8 + i % 12 tokens ((i*31 + j*17) % (vocab-1)) + 1
    and asks for 128 new tokens when i % 5 == 0, else 16."""
    prompts, max_new = [], []
    for i in range(num_requests):
        plen = 8 + i % 12
        prompts.append([((i * 31 + j * 17) % (vocab - 1)) + 1 for j in range(plen)])
        max_new.append(128 if i % 5 == 0 else 16)
    return prompts, max_new


# Model configurations of the token-stream fixtures.
TOY_MODEL = dict(vocab=512, hidden=128, layers=2, heads=4, head_dim=32, ffn=256)
WIDE_MODEL = dict(vocab=32000, hidden=4096, layers=4, heads=32, head_dim=128, ffn=11008)
