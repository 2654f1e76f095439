"""nvllm_paged_attention_static, the entry point that allocates nothing.

It serves callers that cannot allocate device memory (a host that reaches the
GPU only through the C ABI and has no device allocator, or a serving loop whose
memory pool forbids extra cudaMalloc / cudaFree, which synchronize the device
mid-step): the workspace is a 64 MiB array owned by the library on each GPU.

The test calls it through the C ABI twice in a row on the same mixed prefill +
decode batch and compares both outputs with those of the workspace entry point
(nvllm_paged_attention) at the same precision: fp32 prefill tiles within the
fp32 tolerance of the other parity tests, tensor-core prefill tiles,
which lay the shared array out for their 128-row query tiles, within the TF32
tolerance.
It also checks that a batch needing more than 64 MiB of workspace is refused.
This file is collected last so that a run stopping at the first failure has
already run every other test; it builds its own batch and passes alone too.
"""
import ctypes
import math

import numpy as np
import pytest

from helpers import TOL_FP32, TOL_TF32

pytestmark = pytest.mark.gpu

STATIC_WORKSPACE_BYTES = 64 << 20


def _bind(nv):
    f = nv.lib().nvllm_paged_attention_static
    vp, i32 = ctypes.c_void_p, ctypes.c_int32
    f.restype = ctypes.c_int
    f.argtypes = [vp, vp, vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, ctypes.c_float, i32,
                  ctypes.POINTER(nv.KVLayout), vp]
    return f


def _mixed_batch(nv):
    import torch
    dev = torch.device("cuda:0")
    gen = torch.Generator(device=dev)
    gen.manual_seed(31)
    H, hd, B = 32, 128, 16
    rng = np.random.default_rng(31)
    ctx = np.concatenate([[300, 420], rng.integers(100, 3001, 30)]).astype(np.int32)
    ql = np.concatenate([[300, 120], np.ones(30)]).astype(np.int32)
    nbs = (ctx + B - 1) // B
    num_blocks = int(nbs.sum()) + 32
    lay = nv.KVLayout(num_blocks, 1, B, H, hd)
    ka = torch.empty(lay.arena_shape(), device=dev).normal_(generator=gen)
    va = torch.empty_like(ka).normal_(generator=gen)
    perm = rng.permutation(num_blocks).astype(np.int32)
    bt = np.zeros((len(ctx), int(nbs.max())), np.int32)
    off = 0
    for s, nb in enumerate(nbs):
        bt[s, :nb] = perm[off:off + nb]
        off += nb
    cu = np.concatenate([[0], np.cumsum(ql)]).astype(np.int32)
    q = torch.randn((int(cu[-1]), H * hd), generator=gen, device=dev)
    return dict(lay=lay, ka=ka, va=va, q=q, bt=torch.from_numpy(bt).to(dev),
                cu=torch.from_numpy(cu).to(dev), ctx=torch.from_numpy(ctx).to(dev),
                max_q=int(ql.max()), max_ctx=int(ctx.max()), scale=1.0 / math.sqrt(hd))


@pytest.mark.parametrize("precision_name,tol", [("PRECISION_FP32", TOL_FP32),
                                                ("PRECISION_TF32", TOL_TF32)])
def test_no_alloc_entry_point_matches_workspace_entry_point(nv, precision_name, tol):
    import torch
    precision = getattr(nv, precision_name)
    static_attn = _bind(nv)
    b = _mixed_batch(nv)
    lay = b["lay"]
    assert nv.workspace_size(len(b["ctx"]), b["max_q"], b["max_ctx"], lay) <= STATIC_WORKSPACE_BYTES
    ref = torch.full_like(b["q"], float("nan"))
    nv.paged_attention(ref, b["q"], b["ka"], b["va"], b["bt"], b["cu"], b["ctx"], b["max_q"],
                       b["max_ctx"], 0, lay, scale=b["scale"], precision=precision)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(b["q"], float("nan"))
        rc = static_attn(out.data_ptr(), b["q"].data_ptr(), b["ka"].data_ptr(), b["va"].data_ptr(),
                         b["bt"].data_ptr(), b["bt"].shape[1], b["cu"].data_ptr(),
                         b["ctx"].data_ptr(), len(b["ctx"]), b["max_q"], b["max_ctx"], 0,
                         b["scale"], precision, ctypes.byref(lay), stream)
        assert rc == nv.OK, nv.status_string(rc)
        torch.cuda.synchronize()
        assert nv.get_last_error() == nv.OK
        err = (out - ref).abs().max().item()
        assert err <= tol, f"call {call}: max-abs {err} vs the workspace entry point"


def test_no_alloc_entry_point_refuses_oversized_batches(nv):
    import torch
    static_attn = _bind(nv)
    lay = nv.KVLayout(1 << 20, 1, 16, 32, 128)
    # 1024 sequences of up to 65536 positions need far more than 64 MiB of partials
    assert nv.workspace_size(1024, 1, 65536, lay) > STATIC_WORKSPACE_BYTES
    dummy = torch.zeros(64, device="cuda")
    p = dummy.data_ptr()
    rc = static_attn(p, p, p, p, p, 4096, p, p, 1024, 1, 65536, 0, 0.1, nv.PRECISION_FP32,
                     ctypes.byref(lay), torch.cuda.current_stream().cuda_stream)
    assert rc == nv.ERR_WORKSPACE
