"""ctypes binding of libnvllm_host.so (C ABI in include/nvllm_host.h): the
reference-semantics block allocator, the flattened-metadata packer and the
per-device attention engine. Raises if the library is not built."""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import KVLayout, NvllmError, OK, PKG, lib as core_lib

HOST_LIB_PATH = PKG / "lib" / "libnvllm_host.so"
OUT_OF_BLOCKS = 100
INVALID_BLOCK = 101
PACK_ERROR = 102

_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_f32p = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p


class MetadataOffsets(ctypes.Structure):
    _fields_ = [("cu_seqlens_q", ctypes.c_int64), ("context_lens", ctypes.c_int64),
                ("last_token_idx", ctypes.c_int64), ("slot_mapping", ctypes.c_int64),
                ("block_tables", ctypes.c_int64), ("bytes", ctypes.c_int64),
                ("num_seqs", ctypes.c_int32), ("num_tokens", ctypes.c_int32),
                ("max_blocks", ctypes.c_int32), ("max_query_len", ctypes.c_int32),
                ("max_context_len", ctypes.c_int32)]


class EngineConfig(ctypes.Structure):
    _fields_ = [("layout", KVLayout), ("max_seqs", ctypes.c_int32),
                ("max_tokens", ctypes.c_int32), ("max_blocks_per_seq", ctypes.c_int32),
                ("device", ctypes.c_int32)]


class ModelConfig(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int64), ("hidden", ctypes.c_int64), ("layers", ctypes.c_int64),
                ("heads", ctypes.c_int64), ("head_dim", ctypes.c_int64), ("ffn", ctypes.c_int64),
                ("emb_scale", ctypes.c_float), ("ffn_scale", ctypes.c_float)]


_HOST: ctypes.CDLL | None = None


def host_lib() -> ctypes.CDLL:
    global _HOST
    if _HOST is not None:
        return _HOST
    core_lib()  # libnvllm.so first (the host library links against it)
    if not HOST_LIB_PATH.exists():
        raise ImportError(f"{HOST_LIB_PATH} is not built; run `python -m nvllm.build`")
    L = ctypes.CDLL(str(HOST_LIB_PATH))
    L.nvllm_block_allocator_create.restype = _vp
    L.nvllm_block_allocator_create.argtypes = [ctypes.c_int64]
    L.nvllm_block_allocator_destroy.argtypes = [_vp]
    L.nvllm_block_allocator_allocate_block.argtypes = [_vp, _i64p]
    L.nvllm_block_allocator_allocate_blocks.argtypes = [_vp, ctypes.c_int64, _i64p]
    L.nvllm_block_allocator_free_blocks.argtypes = [_vp, _i64p, ctypes.c_int64]
    L.nvllm_block_allocator_num_free.restype = ctypes.c_int64
    L.nvllm_block_allocator_num_free.argtypes = [_vp]
    L.nvllm_metadata_bytes.restype = ctypes.c_size_t
    L.nvllm_metadata_bytes.argtypes = [ctypes.c_int32] * 3
    L.nvllm_pack_metadata.argtypes = [ctypes.c_int32, _i32p, _i32p, _i64p, _i32p, ctypes.c_int32,
                                      ctypes.c_int32, _vp, ctypes.c_size_t,
                                      ctypes.POINTER(MetadataOffsets)]
    L.nvllm_engine_create.argtypes = [ctypes.POINTER(EngineConfig), ctypes.POINTER(_vp)]
    L.nvllm_engine_destroy.argtypes = [_vp]
    L.nvllm_engine_allocate_blocks.argtypes = [_vp, ctypes.c_int64, _i64p]
    L.nvllm_engine_free_blocks.argtypes = [_vp, _i64p, ctypes.c_int64]
    L.nvllm_engine_num_free_blocks.restype = ctypes.c_int64
    L.nvllm_engine_num_free_blocks.argtypes = [_vp]
    L.nvllm_engine_begin_step.argtypes = [_vp, ctypes.c_int32, _i32p, _i32p, _i64p, _i32p]
    L.nvllm_engine_attention.argtypes = [_vp, ctypes.c_int32, _f32p, _f32p, _f32p, _f32p,
                                         ctypes.c_int32]
    L.nvllm_engine_host_buffers.argtypes = [_vp] + [ctypes.POINTER(_f32p)] * 4
    L.nvllm_engine_arenas.argtypes = [_vp, ctypes.POINTER(_f32p), ctypes.POINTER(_f32p)]
    L.nvllm_engine_stream.restype = _vp
    L.nvllm_engine_stream.argtypes = [_vp]
    L.nvllm_engine_step_tokens.restype = ctypes.c_int32
    L.nvllm_engine_step_tokens.argtypes = [_vp]
    L.nvllm_model_create.argtypes = [ctypes.POINTER(ModelConfig), _vp, ctypes.POINTER(_vp)]
    L.nvllm_model_destroy.argtypes = [_vp]
    L.nvllm_model_forward.argtypes = [_vp, _i64p, ctypes.c_int64, _i64p, ctypes.c_int64, _i64p,
                                      ctypes.c_int32, _f32p, _i32p, _f32p, ctypes.c_int32]
    L.nvllm_model_weights.argtypes = [_vp, ctypes.POINTER(_f32p), _i64p]
    _HOST = L
    return L


def _ptr(a, t):
    return a.ctypes.data_as(t)


def _tables(tables):
    """List of per-sequence block-id sequences -> (ids int64, lens int32)."""
    lens = np.array([len(t) for t in tables], np.int32)
    ids = (np.concatenate([np.asarray(t, np.int64) for t in tables]) if len(tables) and lens.sum()
           else np.zeros(1, np.int64))
    return np.ascontiguousarray(ids, np.int64), lens


class BlockAllocator:
    """The reference BlockManager's allocator (src/kv_cache.cpp:23-55)."""

    def __init__(self, num_blocks: int):
        self.L = host_lib()
        self.h = self.L.nvllm_block_allocator_create(num_blocks)
        if not self.h:
            raise ValueError("allocator creation failed")

    def __del__(self):
        if getattr(self, "h", None):
            self.L.nvllm_block_allocator_destroy(self.h)
            self.h = None

    def allocate_block(self):
        out = ctypes.c_int64()
        rc = self.L.nvllm_block_allocator_allocate_block(self.h, ctypes.byref(out))
        return None if rc else out.value

    def allocate_blocks(self, count: int):
        out = np.zeros(max(count, 1), np.int64)
        rc = self.L.nvllm_block_allocator_allocate_blocks(self.h, count, _ptr(out, _i64p))
        return None if rc else out[:count].copy()

    def free_blocks(self, ids) -> int:
        ids = np.ascontiguousarray(ids, np.int64)
        return self.L.nvllm_block_allocator_free_blocks(self.h, _ptr(ids, _i64p), len(ids))

    def num_free(self) -> int:
        return self.L.nvllm_block_allocator_num_free(self.h)


def pack_metadata(num_computed, total_len, tables, block_size: int, max_blocks: int) -> dict:
    """Host packer (no GPU): returns the int32 sections of the packed buffer."""
    L = host_lib()
    nc = np.ascontiguousarray(num_computed, np.int32)
    tl = np.ascontiguousarray(total_len, np.int32)
    ids, lens = _tables(tables)
    S = len(tl)
    n = int((tl - nc).sum()) if S else 0
    nbytes = L.nvllm_metadata_bytes(S, max(n, 0), max_blocks)
    buf = np.zeros(max(nbytes, 16) // 4, np.int32)
    off = MetadataOffsets()
    rc = L.nvllm_pack_metadata(S, _ptr(nc, _i32p), _ptr(tl, _i32p), _ptr(ids, _i64p),
                               _ptr(lens, _i32p), block_size, max_blocks, buf.ctypes.data,
                               buf.nbytes, ctypes.byref(off))
    if rc != OK:
        raise NvllmError(rc, "nvllm_pack_metadata")

    def sec(o, count):
        return buf[o // 4:o // 4 + count].copy()

    return dict(cu_seqlens_q=sec(off.cu_seqlens_q, S + 1), context_lens=sec(off.context_lens, S),
                last_token_idx=sec(off.last_token_idx, S),
                slot_mapping=sec(off.slot_mapping, off.num_tokens),
                block_tables=sec(off.block_tables, S * max_blocks).reshape(S, max_blocks),
                max_query_len=off.max_query_len, max_context_len=off.max_context_len,
                bytes=off.bytes)


class Engine:
    """Per-device attention engine (arenas in HBM, one metadata upload per
    step, host-row attention per layer)."""

    def __init__(self, layout: KVLayout, max_seqs: int, max_tokens: int, max_blocks_per_seq: int,
                 device: int = 0):
        self.L = host_lib()
        self.layout = layout
        cfg = EngineConfig(layout, max_seqs, max_tokens, max_blocks_per_seq, device)
        h = _vp()
        rc = self.L.nvllm_engine_create(ctypes.byref(cfg), ctypes.byref(h))
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_create")
        self.h = h
        self.max_tokens = max_tokens
        bufs = [_f32p() for _ in range(4)]
        self.L.nvllm_engine_host_buffers(self.h, *[ctypes.byref(b) for b in bufs])
        d = layout.hidden
        # numpy views of the engine's pinned row buffers
        self.pinned = [np.ctypeslib.as_array(b, shape=(max_tokens, d)) for b in bufs]

    def close(self):
        if getattr(self, "h", None):
            self.L.nvllm_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def allocate_blocks(self, count: int):
        out = np.zeros(max(count, 1), np.int64)
        rc = self.L.nvllm_engine_allocate_blocks(self.h, count, _ptr(out, _i64p))
        return None if rc else out[:count].copy()

    def free_blocks(self, ids) -> int:
        ids = np.ascontiguousarray(ids, np.int64)
        return self.L.nvllm_engine_free_blocks(self.h, _ptr(ids, _i64p), len(ids))

    def num_free(self) -> int:
        return self.L.nvllm_engine_num_free_blocks(self.h)

    def begin_step(self, num_computed, total_len, tables) -> None:
        nc = np.ascontiguousarray(num_computed, np.int32)
        tl = np.ascontiguousarray(total_len, np.int32)
        ids, lens = _tables(tables)
        rc = self.L.nvllm_engine_begin_step(self.h, len(tl), _ptr(nc, _i32p), _ptr(tl, _i32p),
                                            _ptr(ids, _i64p), _ptr(lens, _i32p))
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_begin_step")

    def prepare_tables(self, tables):
        """Pre-flattened (ids, lens) for begin_step_raw."""
        return _tables(tables)

    def begin_step_raw(self, num_computed, total_len, ids, lens) -> None:
        """begin_step with prepared contiguous int32 / int64 arrays."""
        rc = self.L.nvllm_engine_begin_step(self.h, len(total_len), _ptr(num_computed, _i32p),
                                            _ptr(total_len, _i32p), _ptr(ids, _i64p),
                                            _ptr(lens, _i32p))
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_begin_step")

    def attention(self, layer: int, q, k, v, out, precision: int = 0) -> None:
        for a in (q, k, v, out):
            assert a.dtype == np.float32 and a.flags.c_contiguous
        rc = self.L.nvllm_engine_attention(self.h, layer, _ptr(q, _f32p), _ptr(k, _f32p),
                                           _ptr(v, _f32p), _ptr(out, _f32p), precision)
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_attention")

    def arenas(self):
        k, v = _f32p(), _f32p()
        self.L.nvllm_engine_arenas(self.h, ctypes.byref(k), ctypes.byref(v))
        return ctypes.cast(k, _vp).value, ctypes.cast(v, _vp).value

    def stream(self) -> int:
        return self.L.nvllm_engine_stream(self.h)

    def step_tokens(self) -> int:
        return self.L.nvllm_engine_step_tokens(self.h)


class Model:
    """The reference TransformerModel on the engine's GPU (nvllm_model_*):
    LCG weights generated on the device, forward_batch as device kernels.
    ``cfg`` holds vocab, hidden, layers, heads, head_dim, ffn; ``scales`` the
    optional [emb_scale, ffn_scale] of the weights."""

    def __init__(self, cfg: dict, engine: Engine, scales=None):
        self.L = host_lib()
        self.engine = engine  # the model uses the engine's arenas and stream
        self.cfg = dict(cfg)
        es, fs = (0.0, 0.0) if scales is None else (float(scales[0]), float(scales[1]))
        mc = ModelConfig(cfg["vocab"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["head_dim"],
                         cfg["ffn"], es, fs)
        h = _vp()
        rc = self.L.nvllm_model_create(ctypes.byref(mc), engine.h, ctypes.byref(h))
        if rc != OK:
            raise NvllmError(rc, "nvllm_model_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.L.nvllm_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def forward(self, token_ids, prev_tokens, precision: int = 0, top_k: int = 0):
        """forward_batch over the step begun on the engine. Returns the sampled
        ids, or (sampled, margins, top_idx, top_val) when top_k > 0."""
        tok = np.ascontiguousarray(token_ids, np.int64)
        prev = np.ascontiguousarray(prev_tokens, np.int64)
        s = len(prev)
        sampled = np.zeros(max(s, 1), np.int64)
        margins = np.zeros(max(s, 1), np.float32)
        ti = np.zeros((max(s, 1), max(top_k, 1)), np.int32)
        tv = np.zeros((max(s, 1), max(top_k, 1)), np.float32)
        rc = self.L.nvllm_model_forward(self.h, _ptr(tok, _i64p), len(tok), _ptr(prev, _i64p), s,
                                        _ptr(sampled, _i64p), precision, _ptr(margins, _f32p),
                                        _ptr(ti, _i32p), _ptr(tv, _f32p), top_k)
        if rc != OK:
            raise NvllmError(rc, "nvllm_model_forward")
        if top_k > 0:
            return sampled[:s], margins[:s], ti[:s, :top_k], tv[:s, :top_k]
        return sampled[:s]

    def weights(self) -> tuple[int, int]:
        """(device pointer, float count) of the weight buffer."""
        p, n = _f32p(), ctypes.c_int64()
        rc = self.L.nvllm_model_weights(self.h, ctypes.byref(p), ctypes.byref(n))
        if rc != OK:
            raise NvllmError(rc, "nvllm_model_weights")
        return ctypes.cast(p, _vp).value, n.value
