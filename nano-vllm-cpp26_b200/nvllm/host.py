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


class SchedulerConfig(ctypes.Structure):
    _fields_ = [("max_batch_size", ctypes.c_int64), ("max_tokens_per_step", ctypes.c_int64),
                ("watermark_blocks", ctypes.c_int64), ("eos_token_id", ctypes.c_int64)]


class StepSummary(ctypes.Structure):
    _fields_ = [("admitted", ctypes.c_int64), ("preempted", ctypes.c_int64),
                ("retired", ctypes.c_int64), ("batch_size", ctypes.c_int64),
                ("scheduled_tokens", ctypes.c_int64)]


class Metrics(ctypes.Structure):
    _fields_ = [("uptime_secs", ctypes.c_double), ("total_requests_received", ctypes.c_uint64),
                ("total_requests_completed", ctypes.c_uint64),
                ("total_tokens_generated", ctypes.c_uint64),
                ("throughput_tokens_per_sec", ctypes.c_double),
                ("active_batch_size", ctypes.c_uint64), ("waiting_queue_depth", ctypes.c_uint64),
                ("kv_cache_used_blocks", ctypes.c_uint64),
                ("kv_cache_total_blocks", ctypes.c_uint64),
                ("kv_cache_utilization_pct", ctypes.c_double), ("avg_ttft_ms", ctypes.c_double),
                ("avg_iteration_latency_ms", ctypes.c_double),
                ("total_preemptions", ctypes.c_uint64), ("total_iterations", ctypes.c_uint64),
                ("total_tokens_computed", ctypes.c_uint64), ("h2d_bytes", ctypes.c_uint64),
                ("d2h_bytes", ctypes.c_uint64), ("kernel_launches", ctypes.c_uint64)]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


class ModelConfig(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int64), ("hidden", ctypes.c_int64), ("layers", ctypes.c_int64),
                ("heads", ctypes.c_int64), ("head_dim", ctypes.c_int64), ("ffn", ctypes.c_int64),
                ("emb_scale", ctypes.c_float), ("ffn_scale", ctypes.c_float),
                ("gemm_math", ctypes.c_int32), ("graph_max_tokens", ctypes.c_int32),
                ("head_ranks", ctypes.c_int32)]


class ModelHeadGroup(ctypes.Structure):
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("outs", (ctypes.c_void_p * 8) * 2), ("flags", ctypes.c_void_p * 8)]


GEMM_FP32 = 0
GEMM_BF16X9 = 1
GEMM_TF32X3 = 2


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
    L.nvllm_pack_metadata_padded.argtypes = [ctypes.c_int32, _i32p, _i32p, _i64p, _i32p,
                                             ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                             ctypes.c_int32, _vp, ctypes.c_size_t,
                                             ctypes.POINTER(MetadataOffsets)]
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
    L.nvllm_engine_begin_step_padded.argtypes = [_vp, ctypes.c_int32, _i32p, _i32p, _i64p,
                                                 _i32p, ctypes.c_int32, ctypes.c_int32]
    L.nvllm_engine_attention.argtypes = [_vp, ctypes.c_int32, _f32p, _f32p, _f32p, _f32p,
                                         ctypes.c_int32]
    L.nvllm_engine_host_buffers.argtypes = [_vp] + [ctypes.POINTER(_f32p)] * 4
    L.nvllm_engine_slot_buffers.argtypes = [_vp, ctypes.c_int32] + [ctypes.POINTER(_f32p)] * 4
    L.nvllm_engine_attention_submit.argtypes = [_vp, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_int32]
    L.nvllm_engine_attention_collect.argtypes = [_vp, ctypes.c_int32]
    L.nvllm_router_create.argtypes = [ctypes.POINTER(_vp), ctypes.c_int32, ctypes.POINTER(_vp)]
    L.nvllm_router_destroy.argtypes = [_vp]
    L.nvllm_router_add_request.argtypes = [_vp, ctypes.c_uint64, _i64p, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.POINTER(ctypes.c_int32)]
    L.nvllm_router_add_requests.argtypes = [_vp, ctypes.c_int64,
                                            ctypes.POINTER(ctypes.c_uint64), _i64p, _i64p,
                                            _i64p, _i32p]
    L.nvllm_router_wait_idle.argtypes = [_vp]
    L.nvllm_router_output.restype = ctypes.c_int64
    L.nvllm_router_output.argtypes = [_vp, ctypes.c_uint64, _i64p, ctypes.c_int64]
    L.nvllm_router_metrics.argtypes = [_vp, ctypes.c_int32, ctypes.POINTER(Metrics)]
    L.nvllm_router_placed.restype = ctypes.c_int64
    L.nvllm_router_placed.argtypes = [_vp, ctypes.c_int32]
    L.nvllm_server_start.argtypes = [_vp, ctypes.c_int64, ctypes.c_char_p, ctypes.c_int32,
                                     ctypes.POINTER(_vp)]
    L.nvllm_server_port.restype = ctypes.c_int32
    L.nvllm_server_port.argtypes = [_vp]
    L.nvllm_server_stop.argtypes = [_vp]
    L.nvllm_tokenize_prompt.restype = ctypes.c_int64
    L.nvllm_tokenize_prompt.argtypes = [ctypes.c_char_p, ctypes.c_int64, _i64p, ctypes.c_int64]
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
    L.nvllm_scheduler_create.restype = _vp
    L.nvllm_scheduler_create.argtypes = [ctypes.POINTER(SchedulerConfig), ctypes.c_int32]
    L.nvllm_scheduler_destroy.argtypes = [_vp]
    L.nvllm_scheduler_add_request.argtypes = [_vp, ctypes.c_uint64, _i64p, ctypes.c_int64,
                                              ctypes.c_int64]
    L.nvllm_scheduler_schedule_step.argtypes = [_vp, _vp, ctypes.POINTER(StepSummary)]
    L.nvllm_scheduler_batch_record.restype = ctypes.c_int64
    L.nvllm_scheduler_batch_record.argtypes = [_vp, ctypes.c_int64, _i64p, ctypes.c_int64]
    L.nvllm_scheduler_process_outputs.argtypes = [_vp, _vp, _i64p, ctypes.c_int64, _i64p]
    L.nvllm_scheduler_counts.argtypes = [_vp, _i64p, _i64p, _i64p, _i64p]
    L.nvllm_generator_create.argtypes = [_vp, _vp, ctypes.POINTER(SchedulerConfig),
                                         ctypes.c_int32, ctypes.POINTER(_vp)]
    L.nvllm_generator_destroy.argtypes = [_vp]
    L.nvllm_generator_add_request.argtypes = [_vp, ctypes.c_uint64, _i64p, ctypes.c_int64,
                                              ctypes.c_int64]
    L.nvllm_generator_step.argtypes = [_vp, ctypes.POINTER(StepSummary)]
    L.nvllm_generator_run.argtypes = [_vp, ctypes.c_int64, _i64p]
    L.nvllm_generator_has_pending_work.argtypes = [_vp]
    L.nvllm_generator_output.restype = ctypes.c_int64
    L.nvllm_generator_output.argtypes = [_vp, ctypes.c_uint64, _i64p, ctypes.c_int64]
    L.nvllm_generator_trace.argtypes = [_vp, ctypes.c_char_p]
    L.nvllm_generator_metrics.argtypes = [_vp, ctypes.POINTER(Metrics)]
    L.nvllm_metrics_to_json.restype = ctypes.c_int64
    L.nvllm_metrics_to_json.argtypes = [ctypes.POINTER(Metrics), ctypes.c_char_p, ctypes.c_int64]
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


def pack_metadata(num_computed, total_len, tables, block_size: int, max_blocks: int,
                  pad_seqs: int = 0, pad_tokens: int = 0) -> dict:
    """Host packer (no GPU): returns the int32 sections of the packed buffer
    (laid out as pad_seqs sequences / pad_tokens rows when they are given)."""
    L = host_lib()
    nc = np.ascontiguousarray(num_computed, np.int32)
    tl = np.ascontiguousarray(total_len, np.int32)
    ids, lens = _tables(tables)
    n = int((tl - nc).sum()) if len(tl) else 0
    padded = pad_seqs > 0 or pad_tokens > 0
    S = max(len(tl), pad_seqs)
    nbytes = L.nvllm_metadata_bytes(S, max(n, pad_tokens, 0), max_blocks)
    buf = np.zeros(max(nbytes, 16) // 4, np.int32)
    off = MetadataOffsets()
    if padded:
        rc = L.nvllm_pack_metadata_padded(len(tl), _ptr(nc, _i32p), _ptr(tl, _i32p),
                                          _ptr(ids, _i64p), _ptr(lens, _i32p), block_size,
                                          max_blocks, pad_seqs, pad_tokens, buf.ctypes.data,
                                          buf.nbytes, ctypes.byref(off))
    else:
        rc = L.nvllm_pack_metadata(len(tl), _ptr(nc, _i32p), _ptr(tl, _i32p), _ptr(ids, _i64p),
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

    def begin_step_padded(self, num_computed, total_len, tables, pad_seqs: int,
                          pad_tokens: int) -> None:
        nc = np.ascontiguousarray(num_computed, np.int32)
        tl = np.ascontiguousarray(total_len, np.int32)
        ids, lens = _tables(tables)
        rc = self.L.nvllm_engine_begin_step_padded(self.h, len(tl), _ptr(nc, _i32p),
                                                   _ptr(tl, _i32p), _ptr(ids, _i64p),
                                                   _ptr(lens, _i32p), pad_seqs, pad_tokens)
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_begin_step_padded")

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

    def slot_pinned(self, slot: int):
        """numpy views of a pipeline slot's pinned Q, K, V and output rows
        ([max_tokens, hidden] each; slot 0's are ``pinned``)."""
        bufs = [_f32p() for _ in range(4)]
        rc = self.L.nvllm_engine_slot_buffers(self.h, slot, *[ctypes.byref(b) for b in bufs])
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_slot_buffers")
        d = self.layout.hidden
        return [np.ctypeslib.as_array(b, shape=(self.max_tokens, d)) for b in bufs]

    def submit(self, layer: int, slot: int, precision: int = 0) -> None:
        """Queues the slot's rows through KV write + attention for the step
        begun last (nvllm_engine_attention_submit); returns at once."""
        rc = self.L.nvllm_engine_attention_submit(self.h, layer, slot, precision)
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_attention_submit")

    def collect(self, slot: int) -> None:
        """Waits until the slot's output rows are in its pinned output buffer."""
        rc = self.L.nvllm_engine_attention_collect(self.h, slot)
        if rc != OK:
            raise NvllmError(rc, "nvllm_engine_attention_collect")

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
    optional [emb_scale, ffn_scale] of the weights; ``gemm_math`` GEMM_TF32X3
    (this library's tcgen05 / FFMA GEMMs at fp32 quality; the default where
    hidden, ffn, vocab and hidden / head_ranks are multiples of 128), GEMM_FP32
    (cuBLAS FFMA; the default elsewhere) or GEMM_BF16X9 (cuBLAS's fp32 emulation
    on the tensor cores); ``head_ranks`` > 1 makes it one rank of a
    head-parallel model (the engine holding heads / head_ranks heads; see
    nvllm.headsplit.ModelHeads)."""

    def __init__(self, cfg: dict, engine: Engine, scales=None, gemm_math: int | None = None,
                 graph_max_tokens: int = 0, head_ranks: int = 1):
        if gemm_math is None:
            dims = (cfg["hidden"], cfg["ffn"], cfg["vocab"], cfg["hidden"] // max(head_ranks, 1))
            gemm_math = GEMM_TF32X3 if all(d % 128 == 0 for d in dims) else GEMM_FP32
        self.gemm_math = gemm_math
        self.L = host_lib()
        self.engine = engine  # the model uses the engine's arenas and stream
        self.cfg = dict(cfg)
        es, fs = (0.0, 0.0) if scales is None else (float(scales[0]), float(scales[1]))
        mc = ModelConfig(cfg["vocab"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["head_dim"],
                         cfg["ffn"], es, fs, gemm_math, graph_max_tokens, head_ranks)
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

    def set_head_group(self, rank: int, world: int, outs, flags) -> None:
        """outs[parity][r], flags[r]: device pointers valid in this process."""
        g = ModelHeadGroup()
        g.rank, g.world = rank, world
        for par in range(2):
            for r in range(world):
                g.outs[par][r] = outs[par][r]
        for r in range(world):
            g.flags[r] = flags[r]
        self.L.nvllm_model_set_head_group.argtypes = [_vp, ctypes.POINTER(ModelHeadGroup)]
        rc = self.L.nvllm_model_set_head_group(self.h, ctypes.byref(g))
        if rc != OK:
            raise NvllmError(rc, "nvllm_model_set_head_group")

    def weights(self) -> tuple[int, int]:
        """(device pointer, float count) of the weight buffer."""
        p, n = _f32p(), ctypes.c_int64()
        rc = self.L.nvllm_model_weights(self.h, ctypes.byref(p), ctypes.byref(n))
        if rc != OK:
            raise NvllmError(rc, "nvllm_model_weights")
        return ctypes.cast(p, _vp).value, n.value


def _sched_config(max_batch_size: int, max_tokens_per_step: int, watermark_blocks: int,
                  eos_token_id: int | None) -> SchedulerConfig:
    return SchedulerConfig(max_batch_size, max_tokens_per_step, watermark_blocks,
                           -1 if eos_token_id is None else eos_token_id)


class Scheduler:
    """The continuous-batching scheduler alone (nvllm_scheduler_*), drawing
    blocks from a :class:`BlockAllocator`."""

    def __init__(self, block_size: int, max_batch_size: int = 32, max_tokens_per_step: int = 512,
                 watermark_blocks: int = 4, eos_token_id: int | None = None):
        self.L = host_lib()
        cfg = _sched_config(max_batch_size, max_tokens_per_step, watermark_blocks, eos_token_id)
        self.h = self.L.nvllm_scheduler_create(ctypes.byref(cfg), block_size)
        if not self.h:
            raise NvllmError(1, "nvllm_scheduler_create")

    def __del__(self):
        if getattr(self, "h", None):
            self.L.nvllm_scheduler_destroy(self.h)
            self.h = None

    def add_request(self, seq_id: int, prompt, max_new_tokens: int) -> None:
        p = np.ascontiguousarray(prompt, np.int64)
        rc = self.L.nvllm_scheduler_add_request(self.h, seq_id, _ptr(p, _i64p), len(p),
                                                max_new_tokens)
        if rc != OK:
            raise NvllmError(rc, "nvllm_scheduler_add_request")

    def schedule_step(self, blocks: BlockAllocator) -> dict:
        out = StepSummary()
        rc = self.L.nvllm_scheduler_schedule_step(self.h, blocks.h, ctypes.byref(out))
        if rc != OK:
            raise NvllmError(rc, "nvllm_scheduler_schedule_step")
        return {name: getattr(out, name) for name, _ in StepSummary._fields_}

    def batch_record(self, step: int) -> np.ndarray:
        n = self.L.nvllm_scheduler_batch_record(self.h, step, None, 0)
        out = np.zeros(n, np.int64)
        self.L.nvllm_scheduler_batch_record(self.h, step, _ptr(out, _i64p), n)
        return out

    def process_outputs(self, blocks: BlockAllocator, sampled) -> int:
        smp = np.ascontiguousarray(sampled, np.int64)
        retired = ctypes.c_int64()
        rc = self.L.nvllm_scheduler_process_outputs(self.h, blocks.h, _ptr(smp, _i64p), len(smp),
                                                    ctypes.byref(retired))
        if rc != OK:
            raise NvllmError(rc, "nvllm_scheduler_process_outputs")
        return retired.value

    def counts(self) -> dict:
        v = [ctypes.c_int64() for _ in range(4)]
        self.L.nvllm_scheduler_counts(self.h, *[ctypes.byref(x) for x in v])
        return dict(zip(("running", "waiting", "preemptions", "completed"), (x.value for x in v)))


def metrics_json(m: Metrics) -> str:
    n = host_lib().nvllm_metrics_to_json(ctypes.byref(m), None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    host_lib().nvllm_metrics_to_json(ctypes.byref(m), buf, n + 1)
    return buf.value.decode()


class Generator:
    """The engine loop on one GPU (nvllm_generator_*): scheduler + engine +
    device model."""

    def __init__(self, engine: Engine, model: Model, max_batch_size: int = 32,
                 max_tokens_per_step: int = 512, watermark_blocks: int = 4,
                 eos_token_id: int | None = None, precision: int = 0):
        self.L = host_lib()
        self.engine, self.model = engine, model
        cfg = _sched_config(max_batch_size, max_tokens_per_step, watermark_blocks, eos_token_id)
        h = _vp()
        rc = self.L.nvllm_generator_create(engine.h, model.h, ctypes.byref(cfg), precision,
                                           ctypes.byref(h))
        if rc != OK:
            raise NvllmError(rc, "nvllm_generator_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.L.nvllm_generator_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def add_request(self, seq_id: int, prompt, max_new_tokens: int) -> None:
        p = np.ascontiguousarray(prompt, np.int64)
        rc = self.L.nvllm_generator_add_request(self.h, seq_id, _ptr(p, _i64p), len(p),
                                                max_new_tokens)
        if rc != OK:
            raise NvllmError(rc, "nvllm_generator_add_request")

    def step(self) -> dict:
        out = StepSummary()
        rc = self.L.nvllm_generator_step(self.h, ctypes.byref(out))
        if rc != OK:
            raise NvllmError(rc, "nvllm_generator_step")
        return {name: getattr(out, name) for name, _ in StepSummary._fields_}

    def run(self, max_steps: int = 0) -> int:
        done = ctypes.c_int64()
        rc = self.L.nvllm_generator_run(self.h, max_steps, ctypes.byref(done))
        if rc != OK:
            raise NvllmError(rc, "nvllm_generator_run")
        return done.value

    def has_pending_work(self) -> bool:
        return bool(self.L.nvllm_generator_has_pending_work(self.h))

    def output(self, seq_id: int):
        n = self.L.nvllm_generator_output(self.h, seq_id, None, 0)
        if n < 0:
            return None
        out = np.zeros(n, np.int64)
        self.L.nvllm_generator_output(self.h, seq_id, _ptr(out, _i64p), n)
        return out

    def trace(self, path: str | None) -> None:
        rc = self.L.nvllm_generator_trace(self.h, (path or "").encode())
        if rc != OK:
            raise NvllmError(rc, "nvllm_generator_trace")

    def metrics(self) -> Metrics:
        m = Metrics()
        rc = self.L.nvllm_generator_metrics(self.h, ctypes.byref(m))
        if rc != OK:
            raise NvllmError(rc, "nvllm_generator_metrics")
        return m


class Router:
    """One request stream over several generators (one per GPU), each with its
    own engine thread (nvllm_router_*): requests go to the GPU with the least
    outstanding work. The generators must stay open while the router exists
    and are not to be used directly meanwhile."""

    def __init__(self, generators):
        self.L = host_lib()
        self.generators = list(generators)
        arr = (_vp * len(self.generators))(*[g.h for g in self.generators])
        h = _vp()
        rc = self.L.nvllm_router_create(arr, len(self.generators), ctypes.byref(h))
        if rc != OK:
            raise NvllmError(rc, "nvllm_router_create")
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            self.L.nvllm_router_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def add_request(self, seq_id: int, prompt, max_new_tokens: int) -> int:
        """Places the request; returns the index of the GPU that got it."""
        p = np.ascontiguousarray(prompt, np.int64)
        gpu = ctypes.c_int32()
        rc = self.L.nvllm_router_add_request(self.h, seq_id, _ptr(p, _i64p), len(p),
                                             max_new_tokens, ctypes.byref(gpu))
        if rc != OK:
            raise NvllmError(rc, "nvllm_router_add_request")
        return gpu.value

    def add_requests(self, seq_ids, prompts, max_new_tokens) -> np.ndarray:
        """Places a burst of requests in one call (one decision pass, each GPU
        woken once); returns each request's GPU index. All or nothing."""
        n = len(seq_ids)
        ids = np.ascontiguousarray(seq_ids, np.uint64)
        lens = np.array([len(p) for p in prompts], np.int64)
        offsets = np.zeros(n + 1, np.int64)
        np.cumsum(lens, out=offsets[1:])
        tokens = (np.concatenate([np.asarray(p, np.int64) for p in prompts]) if n
                  else np.zeros(1, np.int64))
        tokens = np.ascontiguousarray(tokens, np.int64)
        mx = np.ascontiguousarray(max_new_tokens, np.int64)
        gpus = np.zeros(max(n, 1), np.int32)
        rc = self.L.nvllm_router_add_requests(
            self.h, n, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
            _ptr(tokens, _i64p), _ptr(offsets, _i64p), _ptr(mx, _i64p), _ptr(gpus, _i32p))
        if rc != OK:
            raise NvllmError(rc, "nvllm_router_add_requests")
        return gpus[:n]

    def wait_idle(self) -> None:
        rc = self.L.nvllm_router_wait_idle(self.h)
        if rc != OK:
            raise NvllmError(rc, "nvllm_router_wait_idle")

    def output(self, seq_id: int):
        n = self.L.nvllm_router_output(self.h, seq_id, None, 0)
        if n < 0:
            return None
        out = np.zeros(n, np.int64)
        self.L.nvllm_router_output(self.h, seq_id, _ptr(out, _i64p), n)
        return out

    def metrics(self, gpu: int) -> Metrics:
        m = Metrics()
        rc = self.L.nvllm_router_metrics(self.h, gpu, ctypes.byref(m))
        if rc != OK:
            raise NvllmError(rc, "nvllm_router_metrics")
        return m

    def placed(self, gpu: int) -> int:
        return self.L.nvllm_router_placed(self.h, gpu)


def tokenize_prompt(text: str, vocab_size: int) -> np.ndarray:
    """The reference engine's prompt tokenisation (nvllm_tokenize_prompt)."""
    L = host_lib()
    raw = text.encode()
    n = L.nvllm_tokenize_prompt(raw, vocab_size, None, 0)
    if n < 0:
        raise NvllmError(1, "nvllm_tokenize_prompt")
    out = np.zeros(n, np.int64)
    L.nvllm_tokenize_prompt(raw, vocab_size, _ptr(out, _i64p), n)
    return out


class Server:
    """The HTTP/SSE front end over a router (nvllm_server_*): GET /health,
    GET /v1/metrics, POST /v1/generate streaming one SSE frame per token.
    Stop it (close) before the router."""

    def __init__(self, router: Router, vocab_size: int, port: int = 0,
                 bind_address: str = "127.0.0.1"):
        self.L = host_lib()
        self.router = router
        h = _vp()
        rc = self.L.nvllm_server_start(router.h, vocab_size, bind_address.encode(), port,
                                       ctypes.byref(h))
        if rc != OK:
            raise NvllmError(rc, "nvllm_server_start")
        self.h = h
        self.port = self.L.nvllm_server_port(h)

    def close(self):
        if getattr(self, "h", None):
            self.L.nvllm_server_stop(self.h)
            self.h = None

    def __del__(self):
        self.close()
