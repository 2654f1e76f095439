"""Python binding of libnvllm.so, the B200 paged-KV write + paged attention
library (C ABI in include/nvllm.h).

Every op calls straight into the CUDA library through ctypes with device
pointers of torch tensors; there is no CPU or eager fallback. If the library
is missing or fails to load, :func:`lib` raises.

Reference correspondence (nano-vllm-cpp26):
  * :func:`reshape_and_cache`  -> the write_kv loop, src/model.cpp:188-202
  * :func:`paged_attention`    -> step 3d of forward_batch, src/model.cpp:204-260
  * :class:`KVLayout`          -> KVCacheConfig, include/nano_vllm/kv_cache.hpp:18-28
"""
from __future__ import annotations

import ctypes
import math
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
LIB_PATH = PKG / "lib" / "libnvllm.so"

OK = 0
ERR_INVALID = 1
ERR_CUDA = 2
ERR_TIMEOUT = 3
ERR_BOUNDS = 4
ERR_WORKSPACE = 5
ERR_UNSUPPORTED = 6

PRECISION_FP32 = 0
PRECISION_TF32 = 1


class NvllmError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = status_string(status) if _LIB is not None else f"status {status}"
        super().__init__(f"{what}: {msg} ({status})" if what else f"{msg} ({status})")


class KVLayout(ctypes.Structure):
    """nvllm_kv_layout: arena [num_blocks, num_layers, block_size, H*hd] fp32."""

    _fields_ = [
        ("num_blocks", ctypes.c_int64),
        ("num_layers", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
    ]

    @property
    def hidden(self) -> int:
        return self.num_heads * self.head_dim

    def arena_shape(self) -> tuple[int, int, int, int]:
        return (self.num_blocks, self.num_layers, self.block_size, self.hidden)

    def __repr__(self) -> str:
        return (f"KVLayout(num_blocks={self.num_blocks}, num_layers={self.num_layers}, "
                f"block_size={self.block_size}, num_heads={self.num_heads}, "
                f"head_dim={self.head_dim})")


MAX_RANKS = 8


class HeadSplit(ctypes.Structure):
    """nvllm_head_split: this rank, the group size, the call's epoch, and every
    rank's output buffer and arrival counter (device pointers valid here)."""

    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("epoch", ctypes.c_uint32),
                ("outs", ctypes.c_void_p * MAX_RANKS), ("flags", ctypes.c_void_p * MAX_RANKS)]


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Loads libnvllm.so (raises if it is not built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built; run `python -m nvllm.build` "
                          "(or __graft_entry__.build())")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, i32, i64, f32, sz = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float,
                             ctypes.c_size_t)
    lp = ctypes.POINTER(KVLayout)
    L.nvllm_reshape_and_cache.restype = ctypes.c_int
    L.nvllm_reshape_and_cache.argtypes = [vp, vp, vp, vp, vp, i64, i32, lp, vp]
    L.nvllm_paged_attention_workspace_size.restype = sz
    L.nvllm_paged_attention_workspace_size.argtypes = [i32, i32, i32, lp]
    L.nvllm_paged_attention.restype = ctypes.c_int
    L.nvllm_paged_attention.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, f32,
                                        i32, vp, sz, lp, vp]
    L.nvllm_paged_attention_head_split.restype = ctypes.c_int
    L.nvllm_paged_attention_head_split.argtypes = [ctypes.POINTER(HeadSplit), vp, vp, vp, vp, i32,
                                                   vp, vp, i32, i32, i32, f32, vp, sz, lp, vp]
    L.nvllm_get_last_error.restype = ctypes.c_int
    L.nvllm_get_last_error.argtypes = [vp]
    L.nvllm_status_string.restype = ctypes.c_char_p
    L.nvllm_status_string.argtypes = [ctypes.c_int]
    _LIB = L
    return L


def status_string(status: int) -> str:
    return lib().nvllm_status_string(status).decode()


def _check(status: int, what: str) -> None:
    if status != OK:
        raise NvllmError(status, what)


def _stream_ptr(stream) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _dptr(t) -> int:
    return t.data_ptr()


def _require(t, dtype_name: str, name: str):
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if str(t.dtype) != f"torch.{dtype_name}":
        raise ValueError(f"{name} must be {dtype_name}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def reshape_and_cache(key, value, k_arena, v_arena, slot_mapping, layer: int,
                      layout: KVLayout, stream=None, check: bool = True) -> int:
    """Writes rows of key/value [n, H*hd] to arena slots (src/model.cpp:188-202)."""
    for t, n, d in ((key, "key", "float32"), (value, "value", "float32"),
                    (k_arena, "k_arena", "float32"), (v_arena, "v_arena", "float32"),
                    (slot_mapping, "slot_mapping", "int32")):
        _require(t, d, n)
    n = slot_mapping.numel()
    st = lib().nvllm_reshape_and_cache(_dptr(key), _dptr(value), _dptr(k_arena), _dptr(v_arena),
                                       _dptr(slot_mapping), n, layer, ctypes.byref(layout),
                                       _stream_ptr(stream))
    if check:
        _check(st, "nvllm_reshape_and_cache")
    return st


def workspace_size(num_seqs: int, max_query_len: int, max_context_len: int,
                   layout: KVLayout) -> int:
    return int(lib().nvllm_paged_attention_workspace_size(num_seqs, max_query_len,
                                                          max_context_len, ctypes.byref(layout)))


def alloc_workspace(num_seqs: int, max_query_len: int, max_context_len: int, layout: KVLayout,
                    device=None):
    import torch
    nbytes = workspace_size(num_seqs, max_query_len, max_context_len, layout)
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device or "cuda")


def paged_attention(out, query, k_arena, v_arena, block_tables, cu_seqlens_q, context_lens,
                    max_query_len: int, max_context_len: int, layer: int, layout: KVLayout,
                    scale: float | None = None, precision: int = PRECISION_FP32, workspace=None,
                    stream=None, check: bool = True) -> int:
    """Causal paged attention over one layer (src/model.cpp:204-260)."""
    for t, n, d in ((out, "out", "float32"), (query, "query", "float32"),
                    (k_arena, "k_arena", "float32"), (v_arena, "v_arena", "float32"),
                    (block_tables, "block_tables", "int32"),
                    (cu_seqlens_q, "cu_seqlens_q", "int32"),
                    (context_lens, "context_lens", "int32")):
        _require(t, d, n)
    num_seqs = context_lens.numel()
    if scale is None:
        scale = 1.0 / math.sqrt(layout.head_dim)
    if workspace is None:
        workspace = alloc_workspace(num_seqs, max_query_len, max_context_len, layout,
                                    device=query.device)
    max_blocks = block_tables.shape[1] if block_tables.dim() == 2 else 1
    st = lib().nvllm_paged_attention(
        _dptr(out), _dptr(query), _dptr(k_arena), _dptr(v_arena), _dptr(block_tables), max_blocks,
        _dptr(cu_seqlens_q), _dptr(context_lens), num_seqs, max_query_len, max_context_len, layer,
        ctypes.c_float(scale), precision, _dptr(workspace), workspace.numel(),
        ctypes.byref(layout), _stream_ptr(stream))
    if check:
        _check(st, "nvllm_paged_attention")
    return st


def get_last_error(stream=None) -> int:
    """Synchronizes and returns/clears the device status word."""
    return lib().nvllm_get_last_error(_stream_ptr(stream))


def paged_attention_head_split(hs: HeadSplit, query, k_arena, v_arena, block_tables,
                               cu_seqlens_q, context_lens, max_context_len: int, layer: int,
                               layout: KVLayout, scale: float | None = None, workspace=None,
                               stream=None, check: bool = True) -> int:
    """Decode attention of this rank's heads; rows land in every rank's output
    buffer (nvllm_paged_attention_head_split)."""
    for t, n, d in ((query, "query", "float32"), (k_arena, "k_arena", "float32"),
                    (v_arena, "v_arena", "float32"), (block_tables, "block_tables", "int32"),
                    (cu_seqlens_q, "cu_seqlens_q", "int32"),
                    (context_lens, "context_lens", "int32")):
        _require(t, d, n)
    num_seqs = context_lens.numel()
    if scale is None:
        scale = 1.0 / math.sqrt(layout.head_dim)
    if workspace is None:
        workspace = alloc_workspace(num_seqs, 1, max_context_len, layout, device=query.device)
    st = lib().nvllm_paged_attention_head_split(
        ctypes.byref(hs), _dptr(query), _dptr(k_arena), _dptr(v_arena), _dptr(block_tables),
        block_tables.shape[1], _dptr(cu_seqlens_q), _dptr(context_lens), num_seqs,
        max_context_len, layer, ctypes.c_float(scale), _dptr(workspace), workspace.numel(),
        ctypes.byref(layout), _stream_ptr(stream))
    if check:
        _check(st, "nvllm_paged_attention_head_split")
    return st
