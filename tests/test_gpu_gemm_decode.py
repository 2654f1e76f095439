"""The two GEMMs of the decode-size projections, both on the weights in the
reference's row-major [k, n] layout and with one signature: nvllm_gemm_skinny
(FFMA, m <= 256) and nvllm_gemm_decode_tc (tcgen05 3xTF32, m <= 32), against a
float64 numpy product: every epilogue, the batched Q/K/V form, row groups
(m > 32, skinny), split-K / stream-K and their fixed order (two runs
bit-identical), K and n tails that are not multiples of the tile, row strides
wider than k, argument errors. The bound: |C - C64| <= 8e-6 * the largest |C64|
of the case (fp32 sums of up to 11008 products; cuBLAS SGEMM on the same cases
errs by up to 4.8e-6)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
REL = 8e-6


IMPLS = ["skinny", "decode_tc"]


def run(m, k, n, batch=1, epilogue=0, lda_pad=0, ldw_pad=0, seed=0, c0=None, want_ws=None,
        impl="skinny"):
    import torch

    import nvllm
    L = nvllm.lib()
    fn = getattr(L, f"nvllm_gemm_{impl}")
    wsf = getattr(L, f"nvllm_gemm_{impl}_workspace_size")
    wsf.restype = ctypes.c_size_t
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k + lda_pad)).astype(np.float32)
    ldw = n + ldw_pad
    w = (rng.standard_normal((batch, k, ldw)) / np.sqrt(k)).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dw = torch.from_numpy(w).cuda()
    init = [np.zeros((m, n), np.float32) if c0 is None else c0[b] for b in range(batch)]
    douts = [torch.from_numpy(np.ascontiguousarray(i)).cuda() for i in init]
    ptrs = (ctypes.c_void_p * batch)(*[t.data_ptr() for t in douts])
    i64 = ctypes.c_int64
    ws_bytes = int(wsf(i64(m), i64(n), i64(k), ctypes.c_int32(batch)))
    if want_ws is not None:
        assert (ws_bytes > 0) == want_ws
    ws = torch.empty(max(ws_bytes, 16) // 4 + 4, dtype=torch.float32, device="cuda")

    def call():
        rc = fn(ctypes.c_void_p(dx.data_ptr()), i64(k + lda_pad), i64(m), i64(k),
                                 ctypes.c_void_p(dw.data_ptr()), i64(ldw), i64(n),
                                 ctypes.c_int32(batch), i64(k * ldw), ptrs, i64(n),
                                 ctypes.c_int32(epilogue), ctypes.c_void_p(ws.data_ptr()),
                                 ctypes.c_size_t(ws.numel() * 4),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == nvllm.OK, nvllm.status_string(rc)
        torch.cuda.synchronize()
        assert nvllm.get_last_error(torch.cuda.current_stream().cuda_stream) == nvllm.OK
        return [t.cpu().numpy() for t in douts]

    got = call()
    errs = []
    for b in range(batch):
        prod = x[:, :k].astype(np.float64) @ w[b, :, :n].astype(np.float64)
        if epilogue == 0:
            want = prod
        elif epilogue == 1:
            want = init[b].astype(np.float64) + prod
        else:
            want = prod / (1.0 + np.exp(-prod))
        errs.append(np.abs(got[b] - want).max() / np.abs(want).max())
    if epilogue == 0:  # the same call again: the fixed-order sums repeat bit for bit
        again = call()
        for b in range(batch):
            assert np.array_equal(again[b], got[b])
    return max(errs), ws_bytes


SHAPES = [
    (1, 128, 128), (3, 96, 256), (8, 4096, 4096), (13, 1024, 640), (26, 4096, 4096),
    (32, 11008, 512), (32, 4096, 11008), (40, 2048, 1024), (77, 1000, 384), (128, 4096, 1024),
    (256, 512, 512),
]


def cases(impl):
    return [s for s in SHAPES if impl == "skinny" or s[0] <= 32]


@pytest.mark.parametrize("impl,m,k,n", [(i,) + s for i in IMPLS for s in cases(i)])
def test_store(impl, m, k, n):
    err, _ = run(m, k, n, impl=impl)
    assert err <= REL, err


@pytest.mark.parametrize("impl", IMPLS)
def test_tails_and_strides(impl):
    # k not a multiple of 32, n not a multiple of 128, padded row strides
    err, _ = run(9, 1001, 300, lda_pad=3, ldw_pad=4, impl=impl)
    assert err <= REL, err
    err, _ = run(31, 70, 132, lda_pad=2, ldw_pad=12, impl=impl)
    assert err <= REL, err
    # n a multiple of 32 but not of 128 (the last tile's atoms past n read as
    # zero), with and without a padded row stride, one matrix and two
    err, _ = run(26, 512, 160, impl=impl)
    assert err <= REL, err
    err, _ = run(17, 300, 224, ldw_pad=32, batch=2, impl=impl)
    assert err <= REL, err


@pytest.mark.parametrize("impl", IMPLS)
def test_split_k_used_for_narrow_outputs(impl):
    err, ws = run(16, 4096, 256, want_ws=True, impl=impl)
    assert ws > 0 and err <= REL, err


@pytest.mark.parametrize("impl", IMPLS)
def test_qkv_batch(impl):
    err, _ = run(20, 1024, 512, batch=3, impl=impl)
    assert err <= REL, err
    err, _ = run(5, 4096, 4096, batch=3, impl=impl)
    assert err <= REL, err


@pytest.mark.parametrize("impl", IMPLS)
def test_accumulate_and_silu(impl):
    rng = np.random.default_rng(7)
    c0 = rng.standard_normal((1, 24, 1024)).astype(np.float32)
    err, _ = run(24, 2048, 1024, epilogue=1, c0=c0, impl=impl)
    assert err <= REL, err
    err, _ = run(24, 2048, 1024, epilogue=2, impl=impl)
    assert err <= REL, err
    m = 64 if impl == "skinny" else 32
    c0 = rng.standard_normal((1, m, 384)).astype(np.float32)
    err, _ = run(m, 4096, 384, epilogue=1, c0=c0, impl=impl)  # split-K then accumulate
    assert err <= REL, err


def test_decode_tc_long_k_does_not_drift():
    """k = 11008 in one tile column: chunked accumulation keeps fp32 quality."""
    err, _ = run(32, 11008, 128, impl="decode_tc")
    assert err <= REL, err


@pytest.mark.parametrize("impl", IMPLS)
def test_argument_errors(impl):
    import nvllm
    L = nvllm.lib()
    fn = getattr(L, f"nvllm_gemm_{impl}")
    wsf = getattr(L, f"nvllm_gemm_{impl}_workspace_size")
    wsf.restype = ctypes.c_size_t
    max_m = 256 if impl == "skinny" else 32
    i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
    outs = (ctypes.c_void_p * 3)(256, 512, 768)
    # (m, k, n, lda, ldw, batch, w_batch_stride): m > 256, lda < k, lda % 4, ldw < n,
    # batch 4, matrices overlapping
    for (m, k, n, lda, ldw, b, wbs) in [(max_m + 1, 64, 128, 64, 128, 1, 0),
                                        (4, 64, 128, 32, 128, 1, 0),
                                        (4, 64, 128, 66, 128, 1, 0), (4, 64, 128, 64, 64, 1, 0),
                                        (4, 64, 128, 64, 128, 4, 8192),
                                        (4, 64, 128, 64, 128, 2, 4096)]:
        rc = fn(vp(256), i64(lda), i64(m), i64(k), vp(256), i64(ldw), i64(n), i32(b), i64(wbs),
                outs, i64(n), i32(0), None, ctypes.c_size_t(0), None)
        assert rc == nvllm.ERR_INVALID, (m, k, n, lda, ldw, b, wbs)
    # a split-K shape without its workspace
    assert wsf(i64(16), i64(256), i64(4096), i32(1)) > 0
    import torch
    x = torch.zeros(16, 4096, device="cuda")
    w = torch.zeros(4096, 256, device="cuda")
    o = torch.zeros(16, 256, device="cuda")
    op = (ctypes.c_void_p * 1)(o.data_ptr())
    rc = fn(vp(x.data_ptr()), i64(4096), i64(16), i64(4096), vp(w.data_ptr()), i64(256), i64(256),
            i32(1), i64(0), op, i64(256), i32(0), None, ctypes.c_size_t(0), None)
    assert rc == nvllm.ERR_WORKSPACE
    assert wsf(i64(0), i64(256), i64(4096), i32(1)) == 0
