"""The device model (nvllm_model_*, nvllm_ops.h) on the GPU:

* each op against numpy on seeded inputs (gathers and the sampler exactly,
  RMSNorm / SiLU / add to fp32 rounding);
* the device LCG weights bit for bit against the oracle's (which is pinned bit
  for bit against the reference's own weights);
* replaying the reference's token traces through the engine + device model:
  every sampled token equal to the reference's, the top-8 LM-head logits within
  LOGIT_RTOL of the reference's values.
"""
import numpy as np
import pytest

from helpers import LOGIT_RTOL, load_trace

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


def _stream(torch):
    return torch.cuda.current_stream().cuda_stream


def _check(nvllm, rc, what):
    assert rc == nvllm.OK, f"{what}: {nvllm.status_string(rc)}"


def test_ops_against_numpy(torch_cuda):
    import ctypes

    import nvllm
    torch = torch_cuda
    L = nvllm.lib()
    vp, i64, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float
    rng = np.random.default_rng(5)
    st = vp(_stream(torch))

    # embedding gather with ids beyond the vocabulary (taken modulo)
    table = rng.standard_normal((50, 36)).astype(np.float32)
    ids = rng.integers(0, 500, 17).astype(np.int32)
    dt, di = torch.from_numpy(table).cuda(), torch.from_numpy(ids).cuda()
    out = torch.full((17, 36), float("nan"), device="cuda")
    _check(nvllm, L.nvllm_embedding_gather(vp(out.data_ptr()), vp(dt.data_ptr()),
                                           vp(di.data_ptr()), i64(17), i64(50), i64(36), st),
           "embedding_gather")
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), table[ids % 50])

    # last-token gather, odd row length (scalar path)
    x = rng.standard_normal((9, 7)).astype(np.float32)
    rows = np.array([8, 0, 3], np.int32)
    dx, dr = torch.from_numpy(x).cuda(), torch.from_numpy(rows).cuda()
    g = torch.zeros((3, 7), device="cuda")
    _check(nvllm, L.nvllm_gather_rows(vp(g.data_ptr()), vp(dx.data_ptr()), vp(dr.data_ptr()),
                                      i64(3), i64(9), i64(7), st), "gather_rows")
    torch.cuda.synchronize()
    assert np.array_equal(g.cpu().numpy(), x[rows])

    # RMSNorm, in place and out of place
    from oracle.model import rms_norm, silu
    for dim in (128, 4096, 30):
        h = (rng.standard_normal((5, dim)) * 3).astype(np.float32)
        dh = torch.from_numpy(h).cuda()
        dn = torch.empty_like(dh)
        _check(nvllm, L.nvllm_rms_norm(vp(dn.data_ptr()), vp(dh.data_ptr()), None, i64(5),
                                       i64(dim), f32(1e-5), st), "rms_norm")
        _check(nvllm, L.nvllm_rms_norm(vp(dh.data_ptr()), vp(dh.data_ptr()), None, i64(5),
                                       i64(dim), f32(1e-5), st), "rms_norm in place")
        torch.cuda.synchronize()
        np.testing.assert_allclose(dn.cpu().numpy(), rms_norm(h), rtol=2e-6, atol=2e-6)
        assert torch.equal(dn, dh)

    # SiLU and add, lengths that are not a multiple of 4
    u = (rng.standard_normal(1003) * 4).astype(np.float32)
    w = rng.standard_normal(1003).astype(np.float32)
    du, dw = torch.from_numpy(u).cuda(), torch.from_numpy(w).cuda()
    _check(nvllm, L.nvllm_silu(vp(du.data_ptr()), i64(1003), st), "silu")
    torch.cuda.synchronize()
    np.testing.assert_allclose(du.cpu().numpy(), silu(u), rtol=2e-6, atol=1e-7)
    du2 = torch.from_numpy(u).cuda()
    _check(nvllm, L.nvllm_add(vp(du2.data_ptr()), vp(dw.data_ptr()), i64(1003), st), "add")
    torch.cuda.synchronize()
    assert np.array_equal(du2.cpu().numpy(), u + w)
    assert nvllm.get_last_error(_stream(torch)) == nvllm.OK


def test_penalized_argmax_against_numpy(torch_cuda):
    import ctypes

    import nvllm
    from oracle.model import penalized_argmax
    torch = torch_cuda
    L = nvllm.lib()
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    rng = np.random.default_rng(9)
    rows, vocab, k = 37, 32000, 8
    logits = rng.standard_normal((rows, vocab)).astype(np.float32)
    # ties (first index wins), a penalised winner, and a row of equal values
    logits[0, 10] = logits[0, 20] = 50.0
    logits[1, 7] = 40.0
    logits[1, 9] = 39.0
    logits[2, :] = 1.0
    prev = rng.integers(0, vocab, rows).astype(np.int64)
    prev[1] = 7
    prev[2] = 5
    prev[3] = vocab + 5  # outside the vocabulary: no penalty
    dl = torch.from_numpy(logits).cuda()
    dp = torch.from_numpy(prev).cuda()
    smp = torch.zeros(rows, dtype=torch.int32, device="cuda")
    mar = torch.zeros(rows, device="cuda")
    ti = torch.zeros((rows, k), dtype=torch.int32, device="cuda")
    tv = torch.zeros((rows, k), device="cuda")
    rc = L.nvllm_penalized_argmax(vp(dl.data_ptr()), vp(dp.data_ptr()), i64(rows), i64(vocab),
                                  ctypes.c_float(1.5), vp(smp.data_ptr()), vp(mar.data_ptr()),
                                  vp(ti.data_ptr()), vp(tv.data_ptr()), ctypes.c_int32(k),
                                  vp(_stream(torch)))
    _check(nvllm, rc, "penalized_argmax")
    torch.cuda.synchronize()
    want, want_margin = penalized_argmax(logits, prev)
    assert np.array_equal(smp.cpu().numpy(), want)
    assert smp[0].item() == 10 and smp[1].item() == 9 and smp[2].item() == 0
    np.testing.assert_array_equal(mar.cpu().numpy(), want_margin)
    order = np.argsort(-logits, axis=1, kind="stable")[:, :k]
    assert np.array_equal(ti.cpu().numpy(), order)
    assert np.array_equal(tv.cpu().numpy(), np.take_along_axis(logits, order, axis=1))


def _device_copy(torch, ptr: int, count: int) -> np.ndarray:
    class View:
        __cuda_array_interface__ = {"shape": (count,), "typestr": "<f4", "data": (ptr, False),
                                    "version": 3}
    return torch.as_tensor(View(), device="cuda").cpu().numpy()


def _engine_for(cfg, z, steps, device_model=True, gemm_math=0):
    import nvllm
    from nvllm.host import Engine, Model
    lay = nvllm.KVLayout(int(z["num_blocks"]), cfg["layers"], int(z["block_size"]), cfg["heads"],
                         cfg["head_dim"])
    max_seqs = max(len(st["seqs"]) for st in steps)
    max_tokens = max(sum(len(s["uncomputed"]) for s in st["seqs"]) for st in steps)
    max_blocks = max(len(s["table"]) for st in steps for s in st["seqs"])
    eng = Engine(lay, max_seqs=max_seqs, max_tokens=max_tokens, max_blocks_per_seq=max_blocks)
    model = Model(cfg, eng, scales=z["scales"][:2], gemm_math=gemm_math) if device_model else None
    return eng, model


def test_device_weights_bit_exact(torch_cuda):
    from oracle.model import model_weights
    cfg, z, steps = load_trace("tokens_toy_seeded")
    eng, model = _engine_for(cfg, z, steps)
    try:
        ptr, count = model.weights()
        got = _device_copy(torch_cuda, ptr, count)
        w = model_weights(cfg, z["scales"])
        flat = [w["embedding"].ravel()]
        for lw in w["layers"]:
            flat += [lw[n].ravel() for n in ("w_q", "w_k", "w_v", "w_o", "w_up", "w_down")]
        flat.append(w["lm_head"].ravel())
        assert np.array_equal(got, np.concatenate(flat))
    finally:
        model.close()
        eng.close()


def replay(name: str, precision: int = 0, gemm_math: int = 0):
    import nvllm
    cfg, z, steps = load_trace(name)
    eng, model = _engine_for(cfg, z, steps, gemm_math=gemm_math)
    try:
        for i, st in enumerate(steps):
            seqs = st["seqs"]
            eng.begin_step([s["num_computed"] for s in seqs], [s["total_len"] for s in seqs],
                           [s["table"] for s in seqs])
            tokens = np.concatenate([s["uncomputed"] for s in seqs])
            prev = np.array([s["prev_token"] for s in seqs], np.int64)
            sampled, margin, ti, tv = model.forward(tokens, prev, precision, top_k=8)
            assert np.array_equal(sampled, st["sampled"]), f"{name} step {i}"
            scale = np.abs(st["top_val"]).max(axis=1, keepdims=True)
            # the reference's top-8 values, and the same indices wherever the
            # reference's neighbouring values are further apart than the tolerance
            assert (np.abs(tv - st["top_val"]) <= LOGIT_RTOL * scale).all(), f"{name} step {i}"
            gap = np.diff(-st["top_val"], axis=1)
            clear = np.concatenate([gap[:, :1], np.minimum(gap[:, 1:], gap[:, :-1]), gap[:, -1:]],
                                   axis=1) > 2 * LOGIT_RTOL * scale
            clear[:, -1] = False  # its lower neighbour is not recorded
            assert (ti[clear] == st["top_idx"][clear]).all(), f"{name} step {i}"
            np.testing.assert_allclose(margin, st["margin"], rtol=0,
                                       atol=2 * LOGIT_RTOL * float(scale.max()))
        assert nvllm.get_last_error(eng.stream()) == nvllm.OK
        return len(steps)
    finally:
        model.close()
        eng.close()


@pytest.mark.parametrize("name", ["tokens_toy_seeded", "tokens_toy_bench", "tokens_wide"])
def test_device_model_replays_reference_tokens(name):
    assert replay(name) > 0


def test_device_model_tf32_attention_wide():
    """The wide model (head_dim 128, block 16) with tcgen05 TF32 prefill tiles:
    the 3xTF32 split keeps the sampled tokens and logits at fp32 quality."""
    assert replay("tokens_wide", precision=1) > 0


@pytest.mark.parametrize("name", ["tokens_toy_seeded", "tokens_toy_bench", "tokens_wide"])
def test_device_model_tcgen05_gemms(name):
    """Projections of more than 32 rows on nvllm_gemm_tf32x3 (3xTF32, fused
    residual / SiLU / Q-K-V epilogues): the reference's tokens and logits."""
    from nvllm.host import GEMM_TF32X3
    assert replay(name, gemm_math=GEMM_TF32X3) > 0


@pytest.mark.parametrize("name", ["tokens_toy_seeded", "tokens_wide"])
def test_device_model_bf16x9_gemms(name):
    """Projections in cuBLAS's bf16x9 emulation of fp32 on the tensor cores:
    the same tokens and the logits within the same fp32 tolerance."""
    import nvllm
    from nvllm.host import GEMM_BF16X9
    try:
        assert replay(name, gemm_math=GEMM_BF16X9) > 0
    except nvllm.NvllmError as e:
        if e.status != nvllm.ERR_UNSUPPORTED:
            raise
        pytest.skip("the cuBLAS loaded in this process has no bf16x9 mode")
