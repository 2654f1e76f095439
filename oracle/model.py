"""Numpy restatement of TransformerModel (src/model.cpp) around the paged
attention path: the LCG weights (:64-112), the embedding gather (:161-166),
RMSNorm (:20-38), the projections (:42-62), SiLU and residual adds (:262-277),
the last-token gather (:280-286), the LM head and the repetition-penalised
greedy sampler (:288-309). The KV write and paged attention go through the C
restatement in nvllm_oracle.c.

Test infrastructure: only the tests use this module, as the checker. It is
pinned against the reference itself: the weights bit for bit against the W
operands the reference's own forward_batch passes to matmul_batched
(``RefPath.model_operands``), the forward against the reference's token traces
(``tests/golden/tokens_*.npz``).
"""
from __future__ import annotations

import numpy as np

from .oracle import KVLayout, Oracle

SEED = 0x5DEECE66D
MUL = 6364136223846793005
MASK = (1 << 64) - 1
PENALTY = np.float32(1.5)   # src/model.cpp:301
RMS_EPS = np.float32(1e-5)  # src/model.cpp:33


def _affine_pow(n: int) -> tuple[int, int]:
    """(a, c) with x -> a*x + c equal to n steps of the LCG x -> MUL*x + 1."""
    ra, rc = 1, 0
    ba, bc = MUL, 1
    while n:
        if n & 1:
            ra, rc = (ba * ra) & MASK, (ba * rc + bc) & MASK
        ba, bc = (ba * ba) & MASK, (ba * bc + bc) & MASK
        n >>= 1
    return ra, rc


def lcg_states(offset: int, count: int) -> np.ndarray:
    """LCG state after draw number offset + i, for i < count (uint64)."""
    out = np.empty(count, np.uint64)
    if count == 0:
        return out
    a, c = _affine_pow(offset + 1)
    out[0] = (a * SEED + c) & MASK
    filled = 1
    with np.errstate(over="ignore"):
        while filled < count:
            n = min(filled, count - filled)
            a, c = _affine_pow(filled)
            out[filled:filled + n] = out[:n] * np.uint64(a) + np.uint64(c)
            filled += n
    return out


def lcg_draws(offset: int, count: int, scale: np.float32) -> np.ndarray:
    """Draws offset .. offset+count-1 of next_f32(scale) (src/model.cpp:74-79)."""
    st = lcg_states(offset, count)
    unit = (st >> np.uint64(33)).astype(np.float32) / np.float32(4294967296.0) - np.float32(0.5)
    return unit * np.float32(scale)


def default_scales(cfg: dict) -> np.ndarray:
    """[emb_scale, ffn_scale, softmax scale] = 1/sqrt(d), 1/sqrt(ffn),
    1/sqrt(head_dim) in fp32, correctly rounded (src/model.cpp:81-82, :205).
    The reference's -ffast-math build may land one unit in the last place
    lower; its own values come from ``RefPath.model_scales`` and are stored in
    the token-trace fixtures."""
    one = np.float32(1.0)
    return np.array([one / np.sqrt(np.float32(cfg[k])) for k in ("hidden", "ffn", "head_dim")],
                    np.float32)


def weight_offsets(cfg: dict) -> dict:
    """Draw index of the first element of every weight, in the constructor's
    order: embedding, per layer w_q, w_k, w_v, w_o, w_up, w_down, then the LM
    head (src/model.cpp:84-112)."""
    v, d, f = cfg["vocab"], cfg["hidden"], cfg["ffn"]
    off = {"embedding": 0}
    pos = v * d
    for layer in range(cfg["layers"]):
        for name, n in (("w_q", d * d), ("w_k", d * d), ("w_v", d * d), ("w_o", d * d),
                        ("w_up", d * f), ("w_down", f * d)):
            off[(layer, name)] = pos
            pos += n
    off["lm_head"] = pos
    off["total"] = pos + d * v
    return off


def model_weights(cfg: dict, scales=None) -> dict:
    v, d, f = cfg["vocab"], cfg["hidden"], cfg["ffn"]
    emb_s, ffn_s = (default_scales(cfg) if scales is None else np.asarray(scales, np.float32))[:2]
    off = weight_offsets(cfg)
    w = {"embedding": lcg_draws(0, v * d, emb_s).reshape(v, d), "layers": []}
    for layer in range(cfg["layers"]):
        lw = {}
        for name, shape in (("w_q", (d, d)), ("w_k", (d, d)), ("w_v", (d, d)), ("w_o", (d, d)),
                            ("w_up", (d, f)), ("w_down", (f, d))):
            sc = ffn_s if name == "w_down" else emb_s
            lw[name] = lcg_draws(off[(layer, name)], shape[0] * shape[1], sc).reshape(shape)
        w["layers"].append(lw)
    w["lm_head"] = lcg_draws(off["lm_head"], d * v, emb_s).reshape(d, v)
    return w


def rms_norm(x: np.ndarray) -> np.ndarray:
    """src/model.cpp:20-38 with weights 1 (the model's rms_attn / rms_ffn)."""
    ss = np.sum(x.astype(np.float64) ** 2, axis=1).astype(np.float32)
    inv = np.float32(1.0) / np.sqrt(ss / np.float32(x.shape[1]) + RMS_EPS)
    return (x * inv[:, None]).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def penalized_argmax(logits: np.ndarray, prev_tokens: np.ndarray):
    """src/model.cpp:293-309: argmax of the logits with PENALTY taken off the
    previous token, lowest index on ties; also the top-2 margin."""
    adj = logits.copy()
    rows = np.arange(len(prev_tokens))
    hit = prev_tokens < logits.shape[1]
    adj[rows[hit], prev_tokens[hit]] -= PENALTY
    sampled = np.argmax(adj, axis=1)  # first maximum
    srt = np.sort(adj, axis=1)
    return sampled, srt[:, -1] - srt[:, -2]


class ModelOracle:
    """Replays forward_batch steps on the CPU with an arena of its own."""

    def __init__(self, cfg: dict, num_blocks: int, block_size: int, scales=None, weights=None):
        self.cfg = cfg
        self.scales = default_scales(cfg) if scales is None else np.asarray(scales, np.float32)
        self.w = weights if weights is not None else model_weights(cfg, self.scales)
        self.lay = KVLayout(num_blocks, cfg["layers"], block_size, cfg["heads"], cfg["head_dim"])
        shape = (num_blocks, cfg["layers"], block_size, cfg["hidden"])
        self.k_arena = np.zeros(shape, np.float32)
        self.v_arena = np.zeros(shape, np.float32)
        self.ora = Oracle()

    def forward(self, seqs: list[dict]):
        """seqs: the running sequences of one step as in a reference trace
        (num_computed, total_len, table, uncomputed, prev_token). Returns the
        sampled ids, the top-2 margins and the LM-head logits."""
        cfg = self.cfg
        v, d = cfg["vocab"], cfg["hidden"]
        B = self.lay.block_size
        nc = np.array([s["num_computed"] for s in seqs], np.int32)
        tl = np.array([s["total_len"] for s in seqs], np.int32)
        fl = self.ora.flatten(nc, tl)
        max_blocks = max(len(s["table"]) for s in seqs)
        bt = np.zeros((len(seqs), max_blocks), np.int32)
        for i, s in enumerate(seqs):
            bt[i, :len(s["table"])] = s["table"]
        slots = self.ora.slot_mapping(fl["cu_seqlens_q"], fl["context_lens"], bt, B)
        tokens = np.concatenate([np.asarray(s["uncomputed"], np.int64) for s in seqs]) % v
        hidden = self.w["embedding"][tokens].copy()
        scale = float(self.scales[2])
        for layer, lw in enumerate(self.w["layers"]):
            x = rms_norm(hidden)
            q, k, vv = x @ lw["w_q"], x @ lw["w_k"], x @ lw["w_v"]
            self.ora.reshape_and_cache(k, vv, self.k_arena, self.v_arena, slots, layer, self.lay)
            attn = self.ora.paged_attention(q, self.k_arena, self.v_arena, bt, fl["cu_seqlens_q"],
                                            fl["context_lens"], layer, scale, self.lay)
            hidden = hidden + attn @ lw["w_o"]
            up = silu(rms_norm(hidden) @ lw["w_up"])
            hidden = hidden + up @ lw["w_down"]
        last = hidden[fl["last_token_idx"]]
        logits = last @ self.w["lm_head"]
        prev = np.array([s["prev_token"] for s in seqs], np.int64)
        sampled, margin = penalized_argmax(logits, prev)
        return sampled, margin, logits
