"""Timing of nvllm_gemm_tf32x3 against cuBLAS fp32 (torch.matmul, TF32 off) on
the projection shapes of the 4096-wide model, decode-size and prefill-size:

    python -m nvllm.gemm_bench [--shapes m,k,n ...] [--reps R] [--once m,k,n]
    python -m nvllm.gemm_bench --skinny [--shapes m,k,n,batch ...] [--once-skinny m,k,n,batch]

For each shape: time per call (CUDA events, after warm-up) with the weights
pre-split into hi / lo (the model's layout) and split on chip, the cuBLAS
time, the error of both against a float64 product. --once runs a single
pre-split call of one shape (for a profiler). --skinny times
nvllm_gemm_skinny (FFMA, decode-size rows, batch weight matrices per call) and
nvllm_gemm_decode_tc (tcgen05, m <= 32) against cuBLAS and the tcgen05 GEMM on
the same shapes, with the weight stream's bandwidth; x cuBLAS is for the
faster of the first two."""
from __future__ import annotations

import argparse
import ctypes

DEFAULT = [(m, k, n) for m in (26, 128) for (k, n) in ((4096, 12288), (4096, 4096), (4096, 11008),
                                                        (11008, 4096), (4096, 32000))] + \
          [(m, k, n) for m in (512, 4096) for (k, n) in ((4096, 12288), (4096, 11008),
                                                         (11008, 4096))]


def main() -> int:
    import torch

    import nvllm
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="*", default=None)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--once", default=None)
    ap.add_argument("--skinny", action="store_true")
    ap.add_argument("--once-skinny", default=None)
    args = ap.parse_args()
    if args.skinny or args.once_skinny:
        return skinny_main(args)
    L = nvllm.lib()
    L.nvllm_gemm_workspace_size.restype = ctypes.c_size_t
    torch.backends.cuda.matmul.allow_tf32 = False
    i64 = ctypes.c_int64

    def setup(m, k, n):
        g = torch.Generator(device="cuda")
        g.manual_seed(m * 31 + k * 7 + n)
        x = torch.randn(m, k, device="cuda", generator=g)
        w = torch.randn(k, n, device="cuda", generator=g) / k ** 0.5
        wt = w.t().contiguous()
        whi, wlo = torch.empty_like(wt), torch.empty_like(wt)
        rc = L.nvllm_tf32_split(ctypes.c_void_p(wt.data_ptr()), ctypes.c_void_p(whi.data_ptr()),
                                ctypes.c_void_p(wlo.data_ptr()), i64(wt.numel()), None)
        assert rc == nvllm.OK
        out = torch.empty(m, n, device="cuda")
        wsb = int(L.nvllm_gemm_workspace_size(i64(m), i64(n), i64(k)))
        ws = torch.empty(max(wsb, 16) // 4 + 4, device="cuda")
        return x, w, wt, whi, wlo, out, ws

    def call(x, m, k, n, hi, lo, out, ws):
        ptrs = (ctypes.c_void_p * 1)(out.data_ptr())
        rc = L.nvllm_gemm_tf32x3(ctypes.c_void_p(x.data_ptr()), i64(k), i64(m), i64(k),
                                 ctypes.c_void_p(hi.data_ptr()),
                                 ctypes.c_void_p(lo.data_ptr() if lo is not None else None),
                                 i64(n), ptrs, ctypes.c_int32(1), i64(n), i64(n),
                                 ctypes.c_int32(0),  # NVLLM_GEMM_STORE
                                 ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws.numel() * 4),
                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == nvllm.OK, nvllm.status_string(rc)

    if args.once:
        m, k, n = (int(v) for v in args.once.split(","))
        x, w, wt, whi, wlo, out, ws = setup(m, k, n)
        call(x, m, k, n, whi, wlo, out, ws)
        torch.cuda.synchronize()
        return 0

    shapes = DEFAULT if not args.shapes else [tuple(int(v) for v in s.split(",")) for s in args.shapes]
    print(f"{'m':>6} {'k':>6} {'n':>6}  {'presplit us':>11} {'TFLOP/s':>8} {'onchip us':>10} "
          f"{'cuBLAS us':>10} {'TFLOP/s':>8} {'x cuBLAS':>8} {'err presplit':>12} {'err cuBLAS':>10}")
    for (m, k, n) in shapes:
        x, w, wt, whi, wlo, out, ws = setup(m, k, n)
        times = {}
        for name, fn in (("pre", lambda: call(x, m, k, n, whi, wlo, out, ws)),
                         ("chip", lambda: call(x, m, k, n, wt, None, out, ws)),
                         ("cublas", lambda: torch.matmul(x, w, out=out))):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            times[name] = e0.elapsed_time(e1) / args.reps * 1e3
        ref = x.double() @ w.double()
        scale = ref.abs().max()
        call(x, m, k, n, whi, wlo, out, ws)
        torch.cuda.synchronize()
        err_pre = ((out.double() - ref).abs().max() / scale).item()
        torch.matmul(x, w, out=out)
        torch.cuda.synchronize()
        err_cb = ((out.double() - ref).abs().max() / scale).item()
        fl = 2.0 * m * k * n
        print(f"{m:6d} {k:6d} {n:6d}  {times['pre']:11.1f} {fl / times['pre'] / 1e6:8.1f} "
              f"{times['chip']:10.1f} {times['cublas']:10.1f} {fl / times['cublas'] / 1e6:8.1f} "
              f"{times['cublas'] / times['pre']:8.2f} {err_pre:12.1e} {err_cb:10.1e}", flush=True)
    assert nvllm.get_last_error(torch.cuda.current_stream().cuda_stream) == nvllm.OK
    return 0


SKINNY = [(m, k, n, b) for m in (1, 8, 16, 26, 32, 48, 64, 96, 128)
          for (k, n, b) in ((4096, 4096, 3), (4096, 4096, 1), (4096, 11008, 1), (11008, 4096, 1),
                            (4096, 32000, 1))]


def skinny_main(args) -> int:
    import torch

    import nvllm
    L = nvllm.lib()
    L.nvllm_gemm_skinny_workspace_size.restype = ctypes.c_size_t
    L.nvllm_gemm_workspace_size.restype = ctypes.c_size_t
    torch.backends.cuda.matmul.allow_tf32 = False
    i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p

    def setup(m, k, n, b):
        g = torch.Generator(device="cuda")
        g.manual_seed(m * 31 + k * 7 + n + b)
        x = torch.randn(m, k, device="cuda", generator=g)
        w = torch.randn(b, k, n, device="cuda", generator=g) / k ** 0.5
        outs = [torch.empty(m, n, device="cuda") for _ in range(b)]
        wsb = max(int(L.nvllm_gemm_skinny_workspace_size(i64(m), i64(n), i64(k), i32(b))),
                  int(L.nvllm_gemm_decode_tc_workspace_size(i64(m), i64(n), i64(k), i32(b))))
        ws = torch.empty(max(wsb, 16) // 4 + 4, device="cuda")
        return x, w, outs, ws

    L.nvllm_gemm_decode_tc_workspace_size.restype = ctypes.c_size_t

    def skinny(x, w, outs, ws, m, k, n, b, fn=L.nvllm_gemm_skinny):
        ptrs = (ctypes.c_void_p * b)(*[o.data_ptr() for o in outs])
        rc = fn(vp(x.data_ptr()), i64(k), i64(m), i64(k), vp(w.data_ptr()), i64(n), i64(n), i32(b),
                i64(k * n), ptrs, i64(n), i32(0), vp(ws.data_ptr()), ctypes.c_size_t(ws.numel() * 4),
                vp(torch.cuda.current_stream().cuda_stream))
        assert rc == nvllm.OK, nvllm.status_string(rc)

    if args.once_skinny:
        m, k, n, b = (int(v) for v in args.once_skinny.split(","))
        x, w, outs, ws = setup(m, k, n, b)
        skinny(x, w, outs, ws, m, k, n, b, fn=L.nvllm_gemm_decode_tc if m <= 32 else L.nvllm_gemm_skinny)
        torch.cuda.synchronize()
        return 0

    shapes = SKINNY if not args.shapes else [tuple(int(v) for v in s.split(",")) for s in args.shapes]
    print(f"{'m':>4} {'k':>6} {'n':>6} {'b':>2}  {'skinny us':>9} {'GB/s':>7} {'TFLOP/s':>7} "
          f"{'dec_tc us':>9} {'GB/s':>7} {'cuBLAS us':>9} {'tf32x3 us':>9} {'x cuBLAS':>8} "
          f"{'err sk':>8} {'err tc':>8}")
    for (m, k, n, b) in shapes:
        x, w, outs, ws = setup(m, k, n, b)
        tc = None
        if b == 1 and n % 128 == 0 and k % 32 == 0:
            wt = w[0].t().contiguous()
            whi, wlo = torch.empty_like(wt), torch.empty_like(wt)
            assert L.nvllm_tf32_split(vp(wt.data_ptr()), vp(whi.data_ptr()), vp(wlo.data_ptr()),
                                      i64(wt.numel()), None) == nvllm.OK
            tws_b = int(L.nvllm_gemm_workspace_size(i64(m), i64(n), i64(k)))
            tws = torch.empty(max(tws_b, 16) // 4 + 4, device="cuda")
            tptr = (ctypes.c_void_p * 1)(outs[0].data_ptr())

            def tc():
                rc = L.nvllm_gemm_tf32x3(vp(x.data_ptr()), i64(k), i64(m), i64(k), vp(whi.data_ptr()),
                                         vp(wlo.data_ptr()), i64(n), tptr, i32(1), i64(n), i64(n),
                                         i32(0), vp(tws.data_ptr()), ctypes.c_size_t(tws.numel() * 4),
                                         vp(torch.cuda.current_stream().cuda_stream))
                assert rc == nvllm.OK

        def cublas():
            for j in range(b):
                torch.matmul(x, w[j], out=outs[j])

        times = {}
        dec = None
        if m <= 32:
            def dec():
                skinny(x, w, outs, ws, m, k, n, b, fn=L.nvllm_gemm_decode_tc)
        for name, fn in (("skinny", lambda: skinny(x, w, outs, ws, m, k, n, b)), ("cublas", cublas),
                         ("tc", tc), ("dec", dec)):
            if fn is None:
                times[name] = float("nan")
                continue
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.reps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            times[name] = e0.elapsed_time(e1) / args.reps * 1e3
        def error(run):
            if run is None:
                return float("nan")
            run()
            torch.cuda.synchronize()
            e = 0.0
            for j in range(b):
                ref = x.double() @ w[j].double()
                e = max(e, ((outs[j].double() - ref).abs().max() / ref.abs().max()).item())
            return e

        err_sk = error(lambda: skinny(x, w, outs, ws, m, k, n, b))
        err_tc = error(dec)
        us, ud = times["skinny"], times["dec"]
        best = min(us, ud) if ud == ud else us
        print(f"{m:4d} {k:6d} {n:6d} {b:2d}  {us:9.1f} {b * k * n * 4 / us / 1e3:7.0f} "
              f"{2.0 * m * k * n * b / us / 1e6:7.1f} {ud:9.1f} {b * k * n * 4 / ud / 1e3:7.0f} "
              f"{times['cublas']:9.1f} {times['tc']:9.1f} {times['cublas'] / best:8.2f} "
              f"{err_sk:8.1e} {err_tc:8.1e}", flush=True)
    assert nvllm.get_last_error(torch.cuda.current_stream().cuda_stream) == nvllm.OK
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
