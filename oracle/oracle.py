"""ctypes front end of the two CPU checkers.

Test infrastructure: only tests, ``__graft_entry__.smoke()`` and the
benchmark's CPU-baseline / reference legs use this module, as the checker.

* :class:`Oracle` wraps ``_build/liboracle.so``, the plain-C restatement of the
  reference algorithm (``nvllm_oracle.c``).
* :class:`RefPath` wraps ``_ref/libref_harness.so``, the reference's own C++
  (``src/kv_cache.cpp``, ``src/model.cpp``, ``src/scheduler.cpp``) built by
  ``make ref``; it exists only where the reference sources were present at build
  time (the built library travels with the tree).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_harness.so"

def reference_sources() -> Path | None:
    """Where the reference's sources lie: ``NVLLM_REFERENCE_DIR`` (no default;
    the reference harness is built only when it names a checkout)."""
    d = os.environ.get("NVLLM_REFERENCE_DIR")
    return Path(d) if d else None

_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)


class KVLayout(ctypes.Structure):
    _fields_ = [
        ("num_blocks", ctypes.c_int64),
        ("num_layers", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
    ]


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def build(with_reference: bool | None = None, reference_dir: Path | str | None = None) -> None:
    """Compile the C oracle and, when the reference sources are present
    (``reference_dir``, else ``NVLLM_REFERENCE_DIR``), the reference harness
    (``make -C oracle [ref] REF=...``)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    src = Path(reference_dir) if reference_dir is not None else reference_sources()
    present = src is not None and (src / "src" / "model.cpp").exists()
    if with_reference is None:
        with_reference = present
    if with_reference:
        if not present:
            raise FileNotFoundError("the reference sources are needed: set NVLLM_REFERENCE_DIR "
                                    "to a checkout of nano-vllm-cpp26")
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={src}"], check=True)


class Oracle:
    """The C restatement (nvllm_oracle.c)."""

    def __init__(self) -> None:
        if not ORACLE_LIB.exists():
            build(with_reference=False)
        lib = ctypes.CDLL(str(ORACLE_LIB))
        lib.oracle_flatten.restype = ctypes.c_int64
        lib.oracle_flatten.argtypes = [ctypes.c_int32, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p, _i32p]
        lib.oracle_slot_mapping.restype = None
        lib.oracle_slot_mapping.argtypes = [ctypes.c_int32, _i32p, _i32p, _i32p, ctypes.c_int32,
                                            ctypes.c_int32, _i32p]
        lib.oracle_reshape_and_cache.restype = None
        lib.oracle_reshape_and_cache.argtypes = [_f32p, _f32p, _f32p, _f32p, _i32p, ctypes.c_int64,
                                                 ctypes.c_int32, ctypes.POINTER(KVLayout)]
        lib.oracle_paged_attention.restype = None
        lib.oracle_paged_attention.argtypes = [
            _f32p, _f32p, _f32p, _f32p, _i32p, ctypes.c_int32, _i32p, _i32p, ctypes.c_int32,
            ctypes.c_int32, ctypes.c_float, ctypes.POINTER(KVLayout), ctypes.c_int32, _u8p,
            ctypes.c_int32]
        self.lib = lib

    def flatten(self, num_computed: np.ndarray, total_len: np.ndarray):
        num_computed = np.ascontiguousarray(num_computed, np.int32)
        total_len = np.ascontiguousarray(total_len, np.int32)
        s = len(total_len)
        n = int((total_len - num_computed).sum())
        cu = np.zeros(s + 1, np.int32)
        ctx = np.zeros(s, np.int32)
        pos = np.zeros(max(n, 1), np.int32)
        seq = np.zeros(max(n, 1), np.int32)
        last = np.zeros(max(s, 1), np.int32)
        got = self.lib.oracle_flatten(s, _ptr(num_computed, _i32p), _ptr(total_len, _i32p),
                                      _ptr(cu, _i32p), _ptr(ctx, _i32p), _ptr(pos, _i32p),
                                      _ptr(seq, _i32p), _ptr(last, _i32p))
        assert got == n
        return dict(cu_seqlens_q=cu, context_lens=ctx, positions=pos[:n], seq_of_token=seq[:n],
                    last_token_idx=last[:s])

    def slot_mapping(self, cu_seqlens_q, context_lens, block_tables, block_size: int) -> np.ndarray:
        cu = np.ascontiguousarray(cu_seqlens_q, np.int32)
        ctx = np.ascontiguousarray(context_lens, np.int32)
        bt = np.ascontiguousarray(block_tables, np.int32)
        out = np.zeros(max(int(cu[-1]), 1), np.int32)
        self.lib.oracle_slot_mapping(len(ctx), _ptr(cu, _i32p), _ptr(ctx, _i32p), _ptr(bt, _i32p),
                                     bt.shape[1], block_size, _ptr(out, _i32p))
        return out[: int(cu[-1])]

    def reshape_and_cache(self, k, v, k_arena, v_arena, slot_mapping, layer: int, lay: KVLayout):
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        sm = np.ascontiguousarray(slot_mapping, np.int32)
        assert k_arena.flags.c_contiguous and v_arena.flags.c_contiguous
        self.lib.oracle_reshape_and_cache(_ptr(k, _f32p), _ptr(v, _f32p), _ptr(k_arena, _f32p),
                                          _ptr(v_arena, _f32p), _ptr(sm, _i32p), len(sm), layer,
                                          ctypes.byref(lay))

    def paged_attention(self, q, k_arena, v_arena, block_tables, cu_seqlens_q, context_lens,
                        layer: int, scale: float, lay: KVLayout, use_f64: bool = False,
                        seq_select=None, num_threads: int = 0, out=None) -> np.ndarray:
        q = np.ascontiguousarray(q, np.float32)
        bt = np.ascontiguousarray(block_tables, np.int32)
        cu = np.ascontiguousarray(cu_seqlens_q, np.int32)
        ctx = np.ascontiguousarray(context_lens, np.int32)
        if out is None:
            out = np.zeros_like(q)
        sel = None
        if seq_select is not None:
            sel = np.ascontiguousarray(seq_select, np.uint8)
        nt = num_threads if num_threads > 0 else (os.cpu_count() or 1)
        self.lib.oracle_paged_attention(
            _ptr(out, _f32p), _ptr(q, _f32p), _ptr(k_arena, _f32p), _ptr(v_arena, _f32p),
            _ptr(bt, _i32p), bt.shape[1], _ptr(cu, _i32p), _ptr(ctx, _i32p), len(ctx), layer,
            ctypes.c_float(scale), ctypes.byref(lay), int(use_f64),
            _ptr(sel, _u8p) if sel is not None else None, nt)
        return out


def reference_available() -> bool:
    return REF_LIB.exists()


class RefPath:
    """The reference's own PagedKVCache + forward_batch, driven through
    ``ref_harness.cpp``."""

    def __init__(self) -> None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} is not built (make -C oracle ref)")
        lib = ctypes.CDLL(str(REF_LIB))
        vp = ctypes.c_void_p
        lib.ref_cache_create.restype = vp
        lib.ref_cache_create.argtypes = [ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_int32, ctypes.c_int32]
        lib.ref_cache_destroy.argtypes = [vp]
        lib.ref_cache_num_free.restype = ctypes.c_int64
        lib.ref_cache_num_free.argtypes = [vp]
        lib.ref_cache_utilization.restype = ctypes.c_double
        lib.ref_cache_utilization.argtypes = [vp]
        lib.ref_cache_allocate_block.restype = ctypes.c_int
        lib.ref_cache_allocate_block.argtypes = [vp, _i64p]
        lib.ref_cache_allocate_blocks.restype = ctypes.c_int
        lib.ref_cache_allocate_blocks.argtypes = [vp, ctypes.c_int64, _i64p]
        lib.ref_cache_free_blocks.argtypes = [vp, _i64p, ctypes.c_int64]
        lib.ref_cache_write_kv.argtypes = [vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                           _f32p, _f32p]
        lib.ref_cache_read_head_kv.argtypes = [vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                               ctypes.c_int32, _f32p, _f32p]
        lib.ref_cache_write_history.argtypes = [vp, ctypes.c_int32, _i32p, _i64p, ctypes.c_int32,
                                                _f32p, _f32p]
        lib.ref_engine_create.restype = vp
        lib.ref_engine_create.argtypes = [ctypes.c_int32] * 4
        lib.ref_generate.restype = ctypes.c_int64
        lib.ref_generate.argtypes = [ctypes.c_int64] * 12 + [_i64p, _i64p, _i64p, ctypes.c_int32,
                                                             ctypes.c_int64, ctypes.c_char_p,
                                                             ctypes.POINTER(ctypes.c_double)]
        lib.ref_inv_sqrt.restype = ctypes.c_float
        lib.ref_inv_sqrt.argtypes = [ctypes.c_float]
        lib.ref_model_operands.restype = ctypes.c_int64
        lib.ref_model_operands.argtypes = [ctypes.c_int64] * 7
        lib.ref_operand_dims.restype = ctypes.c_int
        lib.ref_operand_dims.argtypes = [ctypes.c_int64, _i64p, _i64p, _i64p]
        lib.ref_operand_copy.restype = ctypes.c_int
        lib.ref_operand_copy.argtypes = [ctypes.c_int64, _f32p, _f32p]
        lib.ref_forward_attention.restype = ctypes.c_int64
        lib.ref_forward_attention.argtypes = [vp, vp, ctypes.c_int32, _i32p, _i32p, _i64p,
                                              ctypes.c_int32, _f32p, _f32p, _f32p, _f32p]
        self.lib = lib

    # --- PagedKVCache (src/kv_cache.cpp) -------------------------------------
    def cache_create(self, lay: KVLayout) -> int:
        return self.lib.ref_cache_create(lay.num_blocks, lay.block_size, lay.num_layers,
                                         lay.num_heads, lay.head_dim)

    def cache_destroy(self, c: int) -> None:
        self.lib.ref_cache_destroy(c)

    def num_free(self, c: int) -> int:
        return self.lib.ref_cache_num_free(c)

    def utilization(self, c: int) -> float:
        return self.lib.ref_cache_utilization(c)

    def allocate_block(self, c: int):
        out = ctypes.c_int64(0)
        rc = self.lib.ref_cache_allocate_block(c, ctypes.byref(out))
        return None if rc else out.value

    def allocate_blocks(self, c: int, count: int):
        out = np.zeros(max(count, 1), np.int64)
        rc = self.lib.ref_cache_allocate_blocks(c, count, _ptr(out, _i64p))
        return None if rc else out[:count].copy()

    def free_blocks(self, c: int, ids) -> None:
        ids = np.ascontiguousarray(ids, np.int64)
        self.lib.ref_cache_free_blocks(c, _ptr(ids, _i64p), len(ids))

    def write_kv(self, c: int, block: int, layer: int, slot: int, k, v) -> None:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self.lib.ref_cache_write_kv(c, block, layer, slot, _ptr(k, _f32p), _ptr(v, _f32p))

    def read_head_kv(self, c: int, block: int, layer: int, slot: int, head: int, head_dim: int):
        k = np.zeros(head_dim, np.float32)
        v = np.zeros(head_dim, np.float32)
        self.lib.ref_cache_read_head_kv(c, block, layer, slot, head, _ptr(k, _f32p), _ptr(v, _f32p))
        return k, v

    def write_history(self, c: int, n_prior, block_tables, k, v) -> None:
        n_prior = np.ascontiguousarray(n_prior, np.int32)
        bt = np.ascontiguousarray(block_tables, np.int64)
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        self.lib.ref_cache_write_history(c, len(n_prior), _ptr(n_prior, _i32p), _ptr(bt, _i64p),
                                         bt.shape[1], _ptr(k, _f32p), _ptr(v, _f32p))

    # --- TransformerModel::forward_batch (src/model.cpp:124-312) --------------
    def engine_create(self, num_layers: int, num_heads: int, head_dim: int, num_threads: int = 0) -> int:
        return self.lib.ref_engine_create(num_layers, num_heads, head_dim, num_threads)

    def forward_attention(self, engine: int, cache: int, q_lens, ctx_lens, block_tables,
                          q, k, v, attn_out) -> int:
        q_lens = np.ascontiguousarray(q_lens, np.int32)
        ctx_lens = np.ascontiguousarray(ctx_lens, np.int32)
        bt = np.ascontiguousarray(block_tables, np.int64)
        for a in (q, k, v, attn_out):
            assert a.dtype == np.float32 and a.flags.c_contiguous
        n = self.lib.ref_forward_attention(engine, cache, len(q_lens), _ptr(q_lens, _i32p),
                                           _ptr(ctx_lens, _i32p), _ptr(bt, _i64p), bt.shape[1],
                                           _ptr(q, _f32p), _ptr(k, _f32p), _ptr(v, _f32p),
                                           _ptr(attn_out, _f32p))
        if n < 0:
            raise ValueError("reference harness rejected the batch")
        return n

    # --- continuous batching end to end (src/benchmark.cpp:163-229) -----------
    def generate(self, model: dict, num_blocks: int, block_size: int, max_batch: int,
                 max_tokens_per_step: int, watermark: int, prompts, max_new_tokens,
                 path: str, num_threads: int = 0, max_steps: int = 0) -> list[dict]:
        """Runs the reference scheduler + forward_batch and returns its trace
        (see read_trace)."""
        lens = np.array([len(p) for p in prompts], np.int64)
        toks = np.concatenate([np.asarray(p, np.int64) for p in prompts]) if len(prompts) else \
            np.zeros(1, np.int64)
        mnt = np.asarray(max_new_tokens, np.int64)
        n = self.lib.ref_generate(model["vocab"], model["hidden"], model["layers"], model["heads"],
                                  model["head_dim"], model["ffn"], num_blocks, block_size,
                                  max_batch, max_tokens_per_step, watermark, len(prompts),
                                  _ptr(lens, _i64p), _ptr(np.ascontiguousarray(toks), _i64p),
                                  _ptr(mnt, _i64p), num_threads, max_steps, path.encode(), None)
        if n < 0:
            raise RuntimeError("ref_generate failed")
        return read_trace(path)

    def generate_timed(self, model: dict, num_blocks: int, block_size: int, max_batch: int,
                       max_tokens_per_step: int, watermark: int, prompts, max_new_tokens,
                       num_threads: int = 0) -> tuple[int, float]:
        """The same run without a trace: (steps, seconds of the scheduling
        loop, model construction excluded)."""
        lens = np.array([len(p) for p in prompts], np.int64)
        toks = np.ascontiguousarray(np.concatenate([np.asarray(p, np.int64) for p in prompts]))
        mnt = np.asarray(max_new_tokens, np.int64)
        secs = ctypes.c_double(0.0)
        n = self.lib.ref_generate(model["vocab"], model["hidden"], model["layers"], model["heads"],
                                  model["head_dim"], model["ffn"], num_blocks, block_size,
                                  max_batch, max_tokens_per_step, watermark, len(prompts),
                                  _ptr(lens, _i64p), _ptr(toks, _i64p), _ptr(mnt, _i64p),
                                  num_threads, 0, None, ctypes.byref(secs))
        if n < 0:
            raise RuntimeError("ref_generate failed")
        return int(n), float(secs.value)

    def inv_sqrt(self, x: float) -> np.float32:
        """1.0f / std::sqrt(x) as the reference build evaluates it."""
        return np.float32(self.lib.ref_inv_sqrt(x))

    def model_scales(self, model: dict) -> np.ndarray:
        """[emb_scale, ffn_scale, softmax scale] of the reference build
        (src/model.cpp:81-82, :205)."""
        return np.array([self.inv_sqrt(model["hidden"]), self.inv_sqrt(model["ffn"]),
                         self.inv_sqrt(model["head_dim"])], np.float32)

    def model_operands(self, model: dict, token: int) -> list[tuple[np.ndarray, np.ndarray]]:
        """The (A, W) operands of every matmul_batched call of one reference
        forward_batch over a single one-token sequence: per layer Q, K, V, W_o,
        up, down, then the LM head. The W operands are the model's LCG weights
        as [k, n] matrices."""
        n = self.lib.ref_model_operands(model["vocab"], model["hidden"], model["layers"],
                                        model["heads"], model["head_dim"], model["ffn"], token)
        if n < 0:
            raise RuntimeError("ref_model_operands failed")
        out = []
        for i in range(n):
            b, k, m = (np.zeros(1, np.int64) for _ in range(3))
            self.lib.ref_operand_dims(i, _ptr(b, _i64p), _ptr(k, _i64p), _ptr(m, _i64p))
            a = np.zeros((int(b[0]), int(k[0])), np.float32)
            w = np.zeros((int(k[0]), int(m[0])), np.float32)
            self.lib.ref_operand_copy(i, _ptr(a, _f32p), _ptr(w, _f32p))
            out.append((a, w))
        return out


def read_trace(path_or_array) -> list[dict]:
    """Parses a ref_generate trace (file path or its integer array): one dict
    per step with the running sequences (seq_id, num_computed, total_len,
    prev_token, table, uncomputed), the sampled tokens, the margins and top-8
    logits, and ``record``, the step's raw batch record (header and sequences)."""
    if isinstance(path_or_array, np.ndarray):
        a = path_or_array.astype(np.int64)
    else:
        a = np.fromfile(path_or_array, dtype="<i8")
    i = 0
    steps = []
    while i < len(a):
        start = i
        assert a[i] == -1
        n = int(a[i + 2])
        i += 3
        seqs = []
        for _ in range(n):
            sid, nc, tl, prev, tlen = (int(x) for x in a[i:i + 5])
            i += 5
            table = a[i:i + tlen].copy()
            i += tlen
            nu = int(a[i])
            unc = a[i + 1:i + 1 + nu].copy()
            i += 1 + nu
            seqs.append(dict(seq_id=sid, num_computed=nc, total_len=tl, prev_token=prev,
                             table=table, uncomputed=unc))
        assert a[i] == -2
        record = a[start:i].copy()
        sampled = a[i + 1:i + 1 + n].copy()
        i += 1 + n
        margins = np.zeros(n, np.float32)
        top_idx = np.zeros((n, 8), np.int64)
        top_val = np.zeros((n, 8), np.float32)
        for j in range(n):
            margins[j] = np.array([a[i]], np.int64).astype(np.uint32).view(np.float32)[0]
            pairs = a[i + 1:i + 17].reshape(8, 2)
            top_idx[j] = pairs[:, 0]
            top_val[j] = pairs[:, 1].astype(np.uint32).view(np.float32)
            i += 17
        steps.append(dict(seqs=seqs, sampled=sampled, margin=margins, top_idx=top_idx,
                          top_val=top_val, record=record))
    return steps
