"""Head split of one decode batch across the ranks of a torch.distributed group
(one process per GPU): the output buffers and arrival counters each rank
exposes to its peers through CUDA IPC (libnvllm_host), and the per-call epoch.

Rank r computes heads [r*Hl, (r+1)*Hl); nvllm_paged_attention_head_split
stores every finished row into all ranks' buffers, so after a call each rank's
own buffer holds [n_tokens, world*Hl*hd], the layout of the single-GPU output.
Buffers alternate by epoch parity (a rank cannot overwrite epoch e's rows
before every rank finished epoch e + 1).
"""
from __future__ import annotations

import ctypes

from . import HeadSplit, MAX_RANKS, NvllmError, OK, paged_attention_head_split
from .host import host_lib

HANDLE_BYTES = 64


def _ipc_alloc(nbytes: int):
    L = host_lib()
    L.nvllm_ipc_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(HANDLE_BYTES)
    rc = L.nvllm_ipc_alloc(nbytes, ctypes.byref(ptr), handle)
    if rc != OK:
        raise NvllmError(rc, "nvllm_ipc_alloc")
    return ptr.value, handle.raw


def _ipc_open(handle: bytes) -> int:
    L = host_lib()
    L.nvllm_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
    ptr = ctypes.c_void_p()
    rc = L.nvllm_ipc_open(handle, ctypes.byref(ptr))
    if rc != OK:
        raise NvllmError(rc, "nvllm_ipc_open")
    return ptr.value


class HeadSplitGroup:
    def __init__(self, dist, n_rows: int, local_cols: int, device):
        import torch
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        if self.world > MAX_RANKS:
            raise ValueError(f"head split supports at most {MAX_RANKS} ranks")
        torch.cuda.set_device(device)
        self.device = device
        self.n_rows = n_rows
        self.cols = local_cols * self.world
        nbytes = max(n_rows * self.cols * 4, 256)
        self._own = [_ipc_alloc(nbytes) for _ in range(2)]  # output buffers, by parity
        self._flag = _ipc_alloc(256)
        mine = ([h for _, h in self._own], self._flag[1])
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine)
        self._opened = []
        self.outs = [[0] * self.world for _ in range(2)]
        self.flags = [0] * self.world
        for r, (out_handles, flag_handle) in enumerate(everyone):
            for par in range(2):
                if r == self.rank:
                    self.outs[par][r] = self._own[par][0]
                else:
                    ptr = _ipc_open(out_handles[par])
                    self._opened.append(ptr)
                    self.outs[par][r] = ptr
            if r == self.rank:
                self.flags[r] = self._flag[0]
            else:
                ptr = _ipc_open(flag_handle)
                self._opened.append(ptr)
                self.flags[r] = ptr
        self.epoch = 0
        dist.barrier()

    def output(self, epoch: int | None = None):
        """This rank's gathered output of an epoch (torch view, [n_rows, cols])."""
        import torch
        e = self.epoch if epoch is None else epoch
        ptr = self.outs[e & 1][self.rank]

        class _Mem:
            __cuda_array_interface__ = {"shape": (self.n_rows, self.cols), "typestr": "<f4",
                                        "data": (ptr, False), "version": 3}

        return torch.as_tensor(_Mem(), device=self.device)

    def attention(self, query, k_arena, v_arena, block_tables, cu_seqlens_q, context_lens,
                  max_context_len: int, layer: int, layout, workspace=None, stream=None):
        self.epoch += 1
        hs = HeadSplit()
        hs.rank = self.rank
        hs.world = self.world
        hs.epoch = self.epoch
        for r in range(self.world):
            hs.outs[r] = self.outs[self.epoch & 1][r]
            hs.flags[r] = self.flags[r]
        paged_attention_head_split(hs, query, k_arena, v_arena, block_tables, cu_seqlens_q,
                                   context_lens, max_context_len, layer, layout,
                                   workspace=workspace, stream=stream)
        return self.output()

    def close(self, dist=None):
        import torch
        torch.cuda.synchronize(self.device)
        if dist is not None:
            dist.barrier()  # no peer still writes into our buffers
        L = host_lib()
        L.nvllm_ipc_close.argtypes = [ctypes.c_void_p]
        L.nvllm_ipc_free.argtypes = [ctypes.c_void_p]
        for ptr in self._opened:
            L.nvllm_ipc_close(ptr)
        self._opened = []
        if dist is not None:
            dist.barrier()  # every peer unmapped ours
        for ptr, _ in self._own:
            L.nvllm_ipc_free(ptr)
        L.nvllm_ipc_free(self._flag[0])
        self._own = []


class ModelHeads:
    """The gather buffers of a head-parallel model (nvllm_model_set_head_group):
    two [rows, hidden] fp32 buffers (by epoch parity) and a flag word per rank,
    allocated with nvllm_ipc_alloc and opened in every rank's process."""

    def __init__(self, dist, rows: int, hidden: int, device):
        import torch
        self.rank = dist.get_rank()
        self.world = dist.get_world_size()
        if self.world > MAX_RANKS:
            raise ValueError(f"head parallelism supports at most {MAX_RANKS} ranks")
        torch.cuda.set_device(device)
        nbytes = max(rows * hidden * 4, 256)
        self._own = [_ipc_alloc(nbytes) for _ in range(2)]
        self._flag = _ipc_alloc(256)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, ([h for _, h in self._own], self._flag[1]))
        self._opened = []
        self.outs = [[0] * self.world for _ in range(2)]
        self.flags = [0] * self.world
        for r, (out_handles, flag_handle) in enumerate(everyone):
            for par in range(2):
                if r == self.rank:
                    self.outs[par][r] = self._own[par][0]
                else:
                    self.outs[par][r] = _ipc_open(out_handles[par])
                    self._opened.append(self.outs[par][r])
            if r == self.rank:
                self.flags[r] = self._flag[0]
            else:
                self.flags[r] = _ipc_open(flag_handle)
                self._opened.append(self.flags[r])
        dist.barrier()

    def attach(self, model) -> None:
        model.set_head_group(self.rank, self.world, self.outs, self.flags)

    def close(self, dist=None):
        import torch
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()  # no peer still writes into our buffers
        L = host_lib()
        L.nvllm_ipc_close.argtypes = [ctypes.c_void_p]
        L.nvllm_ipc_free.argtypes = [ctypes.c_void_p]
        for ptr in self._opened:
            L.nvllm_ipc_close(ptr)
        self._opened = []
        if dist is not None:
            dist.barrier()  # every peer unmapped ours
        for ptr, _ in self._own:
            L.nvllm_ipc_free(ptr)
        L.nvllm_ipc_free(self._flag[0])
        self._own = []
