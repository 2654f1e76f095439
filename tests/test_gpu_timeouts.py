"""The bounded device waits give up, report, and leave the GPU usable.

The reference stops the process on a bad block id or row size with an assert
(src/kv_cache.cpp:50-51, :63-64); here every device wait is bounded (2 s of
%globaltimer) and a wait that gives up sets the status word that
nvllm_get_last_error returns as NVLLM_ERR_TIMEOUT, with the kernel's bit in
nvllm_last_status_word and the wait's record in nvllm_last_timeout_info.

Each test makes a cross-GPU flag wait run out on one GPU, with nothing faulted:
a group of one rank whose call's epoch asks for more signals than one rank
sends (world 1, epoch 5: the rank's own signal brings its flag to 1, the wait
wants 5). The call must come back after the 2 s limit with the timeout
reported, and a following call with a reachable target must succeed.
"""
import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TIMEOUT_BIT = 1 << 1
HEAD_GATHER_BIT = 1 << 14
HEAD_SPLIT_BIT = 1 << 15


def _lib(nv):
    L = nv.lib()
    L.nvllm_head_gather.restype = ctypes.c_int
    L.nvllm_head_gather.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.POINTER(nv.HeadSplit), ctypes.c_void_p]
    L.nvllm_last_status_word.restype = ctypes.c_uint32
    L.nvllm_last_timeout_info.restype = ctypes.c_int
    L.nvllm_last_timeout_info.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    return L


def _group_of_one(nv, out, flag, epoch):
    hs = nv.HeadSplit()
    hs.rank, hs.world, hs.epoch = 0, 1, epoch
    hs.outs[0] = out.data_ptr()
    hs.flags[0] = flag.data_ptr()
    return hs


def _timeout_info(L):
    info = (ctypes.c_uint32 * 4)()
    assert L.nvllm_last_timeout_info(info) == 0
    return list(info)


def test_head_gather_wait_gives_up_and_the_next_call_succeeds(nv):
    import torch
    L = _lib(nv)
    assert nv.get_last_error() == nv.OK  # nothing pending from earlier tests
    local = torch.randn(6, 256, device="cuda")
    out = torch.zeros_like(local)
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    hs = _group_of_one(nv, out, flag, epoch=5)
    t0 = time.monotonic()
    assert L.nvllm_head_gather(local.data_ptr(), 6, 256, ctypes.byref(hs), stream) == nv.OK
    st = nv.get_last_error()
    waited = time.monotonic() - t0
    assert st == nv.ERR_TIMEOUT, nv.status_string(st)
    assert 1.9 <= waited < 10.0, f"the wait gave up after {waited:.2f} s, not after ~2 s"
    word = L.nvllm_last_status_word()
    assert word & TIMEOUT_BIT and word & HEAD_GATHER_BIT, hex(word)
    info = _timeout_info(L)
    assert info[0] == HEAD_GATHER_BIT | 1, info
    assert info[1] == 5 and info[3] == 1, info  # awaited 5, read 1 (its own signal)
    # the rows were stored before the wait; the context is intact
    assert torch.equal(out, local)
    assert int(flag.item()) == 1
    # the status was cleared; a call whose target is reachable passes at once
    assert nv.get_last_error() == nv.OK
    hs.epoch = 2  # the signal brings the flag to 2
    out.zero_()
    t0 = time.monotonic()
    assert L.nvllm_head_gather(local.data_ptr(), 6, 256, ctypes.byref(hs), stream) == nv.OK
    assert nv.get_last_error() == nv.OK
    assert time.monotonic() - t0 < 1.0
    assert torch.equal(out, local) and int(flag.item()) == 2


def test_head_split_attention_wait_gives_up_and_the_next_call_succeeds(nv, oracle):
    """nvllm_paged_attention_head_split with a group of one: the attention and
    its row stores complete, the flag wait (epoch 5 with one signal) gives up
    with NVLLM_ERR_TIMEOUT and bit 15; the output is still the attention's, and
    the next call (epoch 2) completes normally."""
    import torch
    from test_gpu_parity import build_batch, oracle_check
    L = _lib(nv)
    assert nv.get_last_error() == nv.OK
    b = build_batch(nv, seed=41, num_blocks=512, block_size=16, num_heads=4, head_dim=128,
                    ctx_lens=[300, 1000, 17], q_lens=[1, 1, 1])
    out = torch.full_like(b["q"], float("nan"))
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    hs = _group_of_one(nv, out, flag, epoch=5)
    ws = nv.alloc_workspace(3, 1, b["max_ctx"], b["lay"], device=b["q"].device)
    t0 = time.monotonic()
    nv.paged_attention_head_split(hs, b["q"], b["ka"], b["va"], b["bt_d"], b["cu_d"], b["ctx_d"],
                                  b["max_ctx"], 0, b["lay"], workspace=ws)
    st = nv.get_last_error()
    waited = time.monotonic() - t0
    assert st == nv.ERR_TIMEOUT, nv.status_string(st)
    assert 1.9 <= waited < 10.0
    word = L.nvllm_last_status_word()
    assert word & TIMEOUT_BIT and word & HEAD_SPLIT_BIT, hex(word)
    info = _timeout_info(L)
    assert info[0] == HEAD_SPLIT_BIT | 1 and info[1] == 5 and info[3] == 1, info
    oracle_check(nv, oracle, b, out, [0, 1, 2])
    hs.epoch = 2
    out.fill_(float("nan"))
    nv.paged_attention_head_split(hs, b["q"], b["ka"], b["va"], b["bt_d"], b["cu_d"], b["ctx_d"],
                                  b["max_ctx"], 0, b["lay"], workspace=ws)
    assert nv.get_last_error() == nv.OK
    assert bool(torch.isfinite(out).all())
    oracle_check(nv, oracle, b, out, [0, 1, 2])
    assert np.int64(flag.item()) == 2
