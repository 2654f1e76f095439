#!/usr/bin/env python3
"""Benchmark of the B200 paged-KV write + paged attention path.

    python bench.py [--gpus N --steps K --warmup W] [--impl nvllm|reference]
                    [--workload decode|mixed|longctx|serve|serve_toy|serve_toy_seeded|
                                serve_router|longctx_model|gemm|gemm_skinny]

One step = one pass of the hot path over one batch: nvllm_reshape_and_cache of
the step's new K/V rows, then nvllm_paged_attention (plan, split-K decode and
merge kernels; the causal prefill kernel too for multi-row sequences). The
default workload is the decode microbenchmark: 64 sequences, contexts
U[512, 4096], 32 heads x head_dim 128, block size 16, 65536-block arena, fp32.

The default line also carries, outside `value`:
  * `e2e`: the same steps through the engine's C ABI with host rows (pinned
    uploads of Q/K/V and metadata, download of the output, two pipeline slots);
  * `sustained`: the step back to back for >= 1.5 s, with its clock record;
  * `parity`: the timed batch's output against the oracle (the C restatement of
    the reference's attention loop), after the timed regions;
  * `extra.mixed`: the mixed prefill + decode super-batch (8 causal prefills
    U[512, 2048] + 120 decodes U[256, 8192]) and its two parts alone;
  * `extra.head_split`: the long-context batch (4 x 32768) with its heads split
    over the ranks (NVLink peer stores) beside the NCCL all-gather variant; at
    N = 1, one rank's share of an N-way split alone for N = 2, 4, 8.
Every timed region has its own clock record (nvidia-smi, the GPU named by UUID).

Under torchrun each rank runs its own batch on its own GPU (sequence
partitioning: the same context lengths in a rank-seeded order and blocks, so
every GPU moves the same bytes; no collective on the data path, weak scaling);
the timed region is bracketed by a barrier and torch.cuda.synchronize(), timed
with CUDA events on the launching stream, and the maximum over ranks is
reported, with every rank's own figures under `per_rank`.

The serving workloads (``serve``, ``serve_toy``, ``serve_toy_seeded``) time the
whole engine loop instead: one step is a complete run of the workload's
requests through the generator (continuous-batching scheduler + device
forward_batch + sampling), reported as output tokens/s; ``serve_router`` runs
one stream of 128 x N requests through the router over N GPUs from one process.
``gemm`` / ``gemm_skinny`` time the model's projection GEMMs (tables on stderr).

``--impl reference`` times the reference's own CPU implementation of the path
(TransformerModel::forward_batch's KV write + paged attention on its
ThreadPool, built from the reference sources into oracle/_ref) on the host
cores, for the same workload and metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "nano-vllm-cpp26_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "paged-attn tokens/s + HBM GB/s (% peak) at 1/2/4/8 B200 vs host-CPU ref"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            pass
    return {}


def profile_traffic(workload: str):
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / f"decode_attention_{workload}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


# ---------------------------------------------------------------------------
# clocks sampled during the timed region


def smi_device_id(local: int) -> str:
    """The name nvidia-smi knows CUDA device ``local`` of this process by: its
    UUID (``GPU-...``), else its PCI bus id. nvidia-smi ignores
    CUDA_VISIBLE_DEVICES, so the process-local ordinal would name whichever GPU
    has that index on the machine, not necessarily this one."""
    import uuid

    import torch
    props = torch.cuda.get_device_properties(local)
    u = getattr(props, "uuid", None)
    if u is not None:
        raw = getattr(u, "bytes", None)
        if isinstance(raw, str):
            raw = raw.encode("latin-1")
        if isinstance(raw, (bytes, bytearray)) and len(raw) == 16:
            return "GPU-" + str(uuid.UUID(bytes=bytes(raw)))
        text = str(u)
        if text:
            return text if text.startswith("GPU-") else "GPU-" + text
    return (f"{int(props.pci_domain_id):08X}:{int(props.pci_bus_id):02X}:"
            f"{int(props.pci_device_id):02X}.0")


class ClockSampler:
    """nvidia-smi clocks, power and throttle reasons of one GPU (named by UUID
    or PCI bus id, see :func:`smi_device_id`), sampled every 50 ms in the
    background between start() and stop()."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_id: str):
        self.device_id = device_id
        self.lines: list[str] = []
        self.stamps: list[float] = []  # time.monotonic() at which each line arrived
        self.proc = None
        self.thread = None

    def command(self) -> list[str]:
        return ["nvidia-smi", f"--id={self.device_id}", f"--query-gpu={self.FIELDS}",
                "--format=csv,noheader,nounits", "-lms", "50"]

    def start(self):
        try:
            self.proc = subprocess.Popen(
                self.command(),
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return self

        def reader():
            for line in self.proc.stdout:
                self.stamps.append(time.monotonic())
                self.lines.append(line.strip())

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        # nvidia-smi takes a while to start: the timed region begins once it samples
        t0 = time.monotonic()
        while not self.lines and self.proc.poll() is None and time.monotonic() - t0 < 5.0:
            time.sleep(0.01)
        return self

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)
        return self.summary(self.lines)

    def window(self, t0: float, t1: float) -> dict:
        """Summary of the samples that arrived between two time.monotonic()
        readings (a timed region; nvidia-smi prints a sample as it takes it)."""
        lines = [ln for ln, t in zip(list(self.lines), list(self.stamps)) if t0 <= t <= t1]
        out = self.summary(lines)
        out["seconds"] = t1 - t0
        return out

    def summary(self, lines) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "device": self.device_id}


# ---------------------------------------------------------------------------
# the reference CPU path


def reference_time(spec, steps: int, warmup: int, budget_s: float | None = None,
                   max_seqs: int | None = None) -> dict:
    """Times the reference's forward_batch (KV write + paged attention; its
    matmuls are answered by the harness) over a batch with the workload's
    shape. The arena holds only the blocks the batch uses (its contents do not
    change the work); tables keep a random permutation."""
    from oracle.oracle import KVLayout, RefPath
    ref = RefPath()
    S = spec.num_seqs if max_seqs is None else min(spec.num_seqs, max_seqs)
    ctx = spec.ctx_lens[:S]
    ql = spec.q_lens[:S]
    B = spec.block_size
    nbs = (ctx + B - 1) // B
    used = int(nbs.sum())
    rng = np.random.Generator(np.random.PCG64(1234))
    perm = rng.permutation(used)
    bt = np.zeros((S, int(nbs.max())), np.int64)
    off = 0
    for s in range(S):
        bt[s, :nbs[s]] = perm[off:off + nbs[s]]
        off += int(nbs[s])
    threads = os.cpu_count() or 1
    lay = KVLayout(used, 1, B, spec.num_heads, spec.head_dim)
    cache = ref.cache_create(lay)
    eng = ref.engine_create(1, spec.num_heads, spec.head_dim, threads)
    n = int(ql.sum())
    D = spec.hidden
    g = np.random.Generator(np.random.PCG64(7))
    q = g.standard_normal((1, n, D), dtype=np.float32)
    k = g.standard_normal((1, n, D), dtype=np.float32)
    v = g.standard_normal((1, n, D), dtype=np.float32)
    out = np.zeros((1, n, D), np.float32)
    for _ in range(max(warmup, 0)):
        ref.forward_attention(eng, cache, ql, ctx, bt, q, k, v, out)
    times = []
    t_start = time.perf_counter()
    for i in range(steps):
        t0 = time.perf_counter()
        ref.forward_attention(eng, cache, ql, ctx, bt, q, k, v, out)
        times.append(time.perf_counter() - t0)
        if budget_s is not None and time.perf_counter() - t_start > budget_s and i >= 1:
            break
    ref.cache_destroy(cache)
    avg = sum(times) / len(times)
    kv = int(ctx.astype(np.int64).sum()) * D * 8
    return {"seconds_per_step": avg, "steps": len(times), "tokens_per_step": n,
            "tokens_per_s": n / avg, "kv_gbs": kv / avg / 1e9, "threads": threads,
            "num_seqs": S, "arena_blocks": used}


def reference_main(args, spec):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.oracle import reference_available
    if not reference_available():
        print(json.dumps({"impl": "reference", "metric": METRIC,
                          "unavailable": "oracle/_ref (the reference's C++ built from its sources) "
                                         "is not present on this machine"}))
        return 0
    # Each step is the full batch unless that would exceed the time budget.
    probe = reference_time(spec, steps=1, warmup=0)
    per = probe["seconds_per_step"]
    max_seqs = None
    budget = 150.0
    if per * (args.steps + args.warmup) > budget:
        frac = budget / (per * (args.steps + args.warmup))
        max_seqs = max(1, int(spec.num_seqs * frac))
    r = reference_time(spec, steps=args.steps, warmup=args.warmup, max_seqs=max_seqs)
    sample = (f"{r['num_seqs']} of {spec.num_seqs} sequences per step, full contexts, "
              f"{r['steps']} timed steps; arena of the {r['arena_blocks']} blocks the batch uses")
    line = {
        "impl": "reference", "metric": METRIC, "value": r["tokens_per_s"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": r["steps"], "warmup": args.warmup,
        "ms_per_step": r["seconds_per_step"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": workload_config(spec),
        "cpu_baseline": {"value": r["tokens_per_s"], "unit": UNIT, "cores": r["threads"],
                         "kind": "reference", "sample": sample, "kv_gbs": r["kv_gbs"]},
        "e2e": {"value": r["tokens_per_s"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def cuda_view(ptr: int, shape, dev):
    """float32 torch tensor over device memory owned elsewhere (the engine)."""
    import torch

    class _Mem:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4",
                                    "data": (ptr, False), "version": 3}

    return torch.as_tensor(_Mem(), device=dev)


def workload_config(spec) -> dict:
    return {"workload": {"decode": "decode paged attention (64 seqs, ctx U[512,4096])",
                         "mixed": "mixed prefill+decode super-batch (8 prefills U[512,2048] "
                                  "+ 120 decodes ctx U[256,8192])",
                         "longctx": "long-context decode (4 seqs x 32768 ctx)",
                         "decode_small": "decode paged attention, profiling size (16 seqs, "
                                         "ctx U[512,4096], 4096-block arena)",
                         "mixed_small": "mixed prefill+decode, profiling size (2 prefills "
                                        "U[512,2048] + 8 decodes, 4096-block arena)"}[spec.name],
            "num_seqs": spec.num_seqs, "num_heads": spec.num_heads, "head_dim": spec.head_dim,
            "block_size": spec.block_size, "arena_blocks": spec.num_blocks,
            "new_tokens_per_step": spec.n_tokens,
            "mean_context": float(spec.ctx_lens.mean()),
            "kv_bytes_per_step": spec.kv_bytes(),
            "l2": "inputs larger than L2 (KV read per step >> 126 MB), no flush"}


# ---------------------------------------------------------------------------
# the nvllm path


class Ranks:
    """The process group around a timed region: barriers, the maximum over
    ranks, gathering per-rank figures. With one process all are no-ops."""

    def __init__(self, dist, dev):
        self.dist, self.dev = dist, dev

    def barrier(self):
        if self.dist is not None:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.dist is None:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, values) -> list[list[float]]:
        """One row of floats per rank, in rank order."""
        import torch
        t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=self.dev)
        if self.dist is None:
            return [t.tolist()]
        out = [torch.empty_like(t) for _ in range(self.dist.get_world_size())]
        self.dist.all_gather(out, t)
        return [o.tolist() for o in out]


def timed_leg(fn, steps: int, warmup: int, stream, ranks: Ranks, sampler, inner=None):
    """W untimed calls of ``fn``, then exactly ``steps`` calls bracketed by a
    barrier and a device synchronize on both sides, timed with CUDA events on
    ``stream``. ``inner(i)`` may return a pair of events to record around
    part of step i. Returns (max-over-ranks seconds, this rank's seconds, the
    clock record of the region)."""
    import torch
    dev = ranks.dev
    for _ in range(warmup):
        fn(None)
    torch.cuda.synchronize(dev)
    ranks.barrier()
    torch.cuda.synchronize(dev)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    t0 = time.monotonic()
    a.record(stream)
    for i in range(steps):
        fn(i)
    b.record(stream)
    torch.cuda.synchronize(dev)
    t1 = time.monotonic()
    ranks.barrier()
    mine = a.elapsed_time(b) / 1e3
    return ranks.max(mine), mine, sampler.window(t0, t1)


class DeviceBatch:
    """A :class:`nvllm.workload.BatchSpec` on the device over given arenas:
    Q/K/V rows of the step's new tokens (N(0,1) from ``gen``), metadata, output
    and workspace; ``step()`` is one pass of the hot path (KV write of the new
    rows + paged attention)."""

    def __init__(self, nvllm, spec, lay, ka, va, gen, dev, stream, precision):
        import torch
        self.nv, self.spec, self.lay, self.ka, self.va = nvllm, spec, lay, ka, va
        self.stream, self.precision = stream, precision
        n, D = spec.n_tokens, lay.num_heads * lay.head_dim  # this GPU's heads
        self.q = torch.randn((n, D), generator=gen, device=dev)
        self.k = torch.randn((n, D), generator=gen, device=dev)
        self.v = torch.randn((n, D), generator=gen, device=dev)
        self.out = torch.empty_like(self.q)
        self.bt = torch.from_numpy(spec.block_tables).to(dev)
        self.cu = torch.from_numpy(spec.cu_seqlens_q).to(dev)
        self.ctx = torch.from_numpy(spec.ctx_lens).to(dev)
        self.slots = torch.from_numpy(spec.slot_mapping()).to(dev)
        self.max_q = int(spec.q_lens.max())
        self.max_ctx = int(spec.ctx_lens.max())
        self.ws = nvllm.alloc_workspace(spec.num_seqs, self.max_q, self.max_ctx, lay, device=dev)

    def write(self):
        self.nv.reshape_and_cache(self.k, self.v, self.ka, self.va, self.slots, 0, self.lay,
                                  stream=self.stream)

    def attend(self, precision=None):
        p = self.precision if precision is None else precision
        self.nv.paged_attention(self.out, self.q, self.ka, self.va, self.bt, self.cu, self.ctx,
                                self.max_q, self.max_ctx, 0, self.lay, workspace=self.ws,
                                stream=self.stream, precision=p)

    def step(self, precision=None):
        self.write()
        self.attend(precision)

    def launches(self) -> int:
        """This library's kernels per step: KV write, plan, decode, merge, and
        the prefill kernel when a sequence has several query rows."""
        return 4 + (1 if self.max_q > 1 else 0)


def oracle_parity(db, seqs, host_budget: int = 2 << 30) -> dict:
    """The step's output rows of ``seqs`` against the oracle (the C restatement
    of the reference's attention loop), from host copies of the blocks those
    sequences read, in groups of at most ``host_budget`` bytes. A check only:
    it runs after the timed regions."""
    import torch

    from oracle.oracle import KVLayout, Oracle
    orc = Oracle()
    spec, lay = db.spec, db.lay
    nbs = (spec.ctx_lens + spec.block_size - 1) // spec.block_size
    row_bytes = 2 * spec.block_size * spec.hidden * 4
    cu = spec.cu_seqlens_q
    groups, cur, blocks = [], [], 0
    for s in seqs:
        if cur and (blocks + int(nbs[s])) * row_bytes > host_budget:
            groups.append(cur)
            cur, blocks = [], 0
        cur.append(int(s))
        blocks += int(nbs[s])
    if cur:
        groups.append(cur)
    worst, rows = 0.0, 0
    for g in groups:
        used = np.unique(np.concatenate([spec.block_tables[s, :nbs[s]] for s in g]))
        remap = np.full(int(used.max()) + 1, -1, np.int64)
        remap[used] = np.arange(len(used))
        idx = torch.from_numpy(used.astype(np.int64)).to(db.ka.device)
        ka = db.ka.index_select(0, idx).cpu().numpy()
        va = db.va.index_select(0, idx).cpu().numpy()
        bt = np.zeros((len(g), spec.block_tables.shape[1]), np.int32)
        q_rows, gcu = [], [0]
        for j, s in enumerate(g):
            bt[j, :nbs[s]] = remap[spec.block_tables[s, :nbs[s]]]
            q_rows.extend(range(int(cu[s]), int(cu[s + 1])))
            gcu.append(len(q_rows))
        ridx = torch.as_tensor(q_rows, device=db.q.device)
        q = db.q.index_select(0, ridx).cpu().numpy()
        got = db.out.index_select(0, ridx).cpu().numpy()
        olay = KVLayout(len(used), 1, spec.block_size, spec.num_heads, spec.head_dim)
        ref = orc.paged_attention(q, ka, va, bt, np.array(gcu, np.int32),
                                  spec.ctx_lens[g].astype(np.int32), 0,
                                  1.0 / math.sqrt(spec.head_dim), olay)
        worst = max(worst, float(np.abs(got - ref).max()))
        rows += len(q_rows)
    return {"max_abs": worst, "rows": rows, "seqs": len(seqs)}


def nvllm_main(args, spec):
    import torch
    import nvllm
    from nvllm.workload import make_batch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    ranks = Ranks(dist, dev)
    nvllm.lib()  # fails loudly when the CUDA library is missing

    # per-rank batch (sequence partitioning): the same context lengths on every
    # GPU, in a rank-seeded order with rank-seeded block tables and values
    heads = spec.num_heads  # fewer than the workload's with --head-slice
    spec = make_batch(args.workload, seed=args.seed, rank=rank)
    if heads != spec.num_heads:
        import dataclasses
        spec = dataclasses.replace(spec, num_heads=heads)
    lay = nvllm.KVLayout(spec.num_blocks, 1, spec.block_size, spec.num_heads, spec.head_dim)
    D = spec.hidden
    # The arenas belong to the host engine (libnvllm_host: allocator, pinned
    # metadata upload, host-row attention); the device-resident loop drives the
    # kernels on the same arenas through libnvllm's C ABI.
    from nvllm.host import Engine
    eng = Engine(lay, max_seqs=spec.num_seqs, max_tokens=spec.n_tokens,
                 max_blocks_per_seq=spec.block_tables.shape[1], device=local)
    k_ptr, v_ptr = eng.arenas()
    ka = cuda_view(k_ptr, lay.arena_shape(), dev)
    va = cuda_view(v_ptr, lay.arena_shape(), dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    ka.normal_(generator=gen)
    va.normal_(generator=gen)
    stream = torch.cuda.current_stream(dev)
    precision = nvllm.PRECISION_TF32 if args.precision == "tf32" else nvllm.PRECISION_FP32
    db = DeviceBatch(nvllm, spec, lay, ka, va, gen, dev, stream, precision)
    n = spec.n_tokens
    warm = max(args.warmup, 3)
    launches = 0

    sampler = ClockSampler(smi_device_id(local)).start()
    t_first = time.monotonic()

    # ---- device-resident throughput --------------------------------------
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]

    def step(i):
        db.write()
        if i is not None:
            ev[i][0].record(stream)
        db.attend()
        if i is not None:
            ev[i][1].record(stream)

    elapsed_max, elapsed_mine, clocks_dev = timed_leg(step, args.steps, warm, stream, ranks,
                                                      sampler)
    launches += db.launches() * args.steps
    if nvllm.get_last_error(stream) != nvllm.OK:
        raise RuntimeError("device status after the timed steps is not OK")
    attn_mine = sum(a.elapsed_time(b) for a, b in ev) / 1e3 / args.steps
    alg_bytes = spec.decode_algorithmic_bytes()

    # ---- end to end through the engine's C ABI with host buffers ---------
    # per step: pack + one pinned upload of the metadata, H2D of the Q/K/V rows
    # from pinned host memory, KV write + attention, D2H of the output into
    # pinned host memory. Steps alternate between the engine's two pipeline
    # slots, so step i+1's copies overlap step i's kernels; the last step's
    # output is collected inside the timed region.
    torch.cuda.synchronize(dev)
    slots = [eng.slot_pinned(0), eng.slot_pinned(1)]
    for h_q, h_k, h_v, _ in slots:
        h_q[:n] = db.q.cpu().numpy()
        h_k[:n] = db.k.cpu().numpy()
        h_v[:n] = db.v.cpu().numpy()
    nc = np.ascontiguousarray(spec.ctx_lens - spec.q_lens, np.int32)
    tl = np.ascontiguousarray(spec.ctx_lens, np.int32)
    nbs = (spec.ctx_lens + spec.block_size - 1) // spec.block_size
    ids, lens = eng.prepare_tables([spec.block_tables[s_, :nbs[s_]] for s_ in range(spec.num_seqs)])
    from nvllm.host import host_lib
    meta_bytes = int(host_lib().nvllm_metadata_bytes(spec.num_seqs, n, spec.block_tables.shape[1]))
    h2d = meta_bytes + 3 * n * D * 4
    d2h = n * D * 4
    estream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    pending = []

    def e2e_drain():
        while pending:
            eng.collect(pending.pop(0))

    def e2e_step(i):
        slot = 0 if not pending else 1 - pending[-1]
        if len(pending) == 2:  # the slot about to be refilled: its output must be back
            eng.collect(pending.pop(0))
        eng.begin_step_raw(nc, tl, ids, lens)
        eng.submit(0, slot, precision)
        pending.append(slot)
        if i == args.steps - 1:  # the timed region ends with the last output on the host
            e2e_drain()

    for _ in range(warm):
        e2e_step(None)
    e2e_drain()
    e2e_elapsed, _, clocks_e2e = timed_leg(e2e_step, args.steps, 0, estream, ranks, sampler)
    e2e_drain()
    launches += db.launches() * args.steps
    status = nvllm.get_last_error(stream)
    if status != nvllm.OK:
        raise RuntimeError(f"device status {nvllm.status_string(status)}")
    h_out = slots[(args.steps - 1) % 2][3][:n]
    e2e_diff = float(np.abs(h_out - db.out.cpu().numpy()).max())

    # ---- the same step back to back for >= 1.5 s: a clock record of sustained
    # load (after the timed legs, so that they start from the same thermal state)
    sus_steps = int(min(20000, max(args.steps, math.ceil(1.5 / max(elapsed_mine / args.steps,
                                                                    1e-6)))))
    sus_steps = int(ranks.max(sus_steps))
    sus_max, _, clocks_sus = timed_leg(lambda i: db.step(), sus_steps, 0, stream, ranks,
                                       sampler)
    launches_sus = db.launches() * sus_steps


    # ---- parity of the timed batch, after its timed regions and before the
    # other batches below write into the same arenas
    parity = None
    if not args.no_parity:
        seqs = list(range(spec.num_seqs)) if world == 1 else list(range(0, spec.num_seqs, 8))
        pr = oracle_parity(db, seqs)
        worst = ranks.max(pr["max_abs"])
        # tensor-core prefill tiles (two-term bf16 products) are held to 1e-3,
        # everything in fp32 to 2e-5
        tol = 1e-3 if precision == nvllm.PRECISION_TF32 and db.max_q > 1 else 2e-5
        parity = {"max_abs": worst, "tol": tol, "ok": worst <= tol,
                  "rows_per_rank": pr["rows"], "seqs_per_rank": pr["seqs"],
                  "e2e_output_max_abs_vs_device_output": ranks.max(e2e_diff),
                  "oracle": "C restatement of the reference's attention loop, on the output "
                            "of the last timed step"}

    # ---- the other benchmark batches (outside `value`) --------------------
    extra = {}
    if args.workload == "decode" and not args.no_extra:
        extra["mixed"] = mixed_leg(args, nvllm, lay, ka, va, dev, stream, ranks, sampler, rank)
        extra["head_split"] = headsplit_leg(args, nvllm, dev, stream, ranks, sampler, rank,
                                            world)
    t_last = time.monotonic()
    clocks_all = sampler.window(t_first, t_last)
    sampler.stop()

    # ---- per-rank figures; the roofline from the slowest rank's own bytes --
    per_rank = ranks.gather([alg_bytes, elapsed_mine, attn_mine])
    slow = max(range(len(per_rank)), key=lambda r: per_rank[r][2])
    attn_max = per_rank[slow][2]
    achieved = per_rank[slow][0] / attn_max / 1e9
    tokens = n * args.steps * world
    value = tokens / elapsed_max
    e2e_value = tokens / e2e_elapsed
    peaks = measured_peaks()
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    if not peak:
        peak = FALLBACK_HBM_GBS

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_max / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic", "config": workload_config(spec),
        "parallelism": f"sequence-partitioned x{world} (equal KV bytes per GPU)",
        "prefill_precision": args.precision,
        "hbm_gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "kernel": "nvllm_paged_attention (plan + split-K decode + merge)",
                     "algorithmic_bytes_per_launch": per_rank[slow][0],
                     "ms_per_launch": attn_max * 1e3, "rank": slow,
                     "traffic": profile_traffic(spec.name)},
        "per_rank": [{"rank": r, "algorithmic_bytes": b_, "ms_per_step": t_ / args.steps * 1e3,
                      "attention_ms": a_ * 1e3, "hbm_frac": b_ / a_ / 1e9 / peak}
                     for r, (b_, t_, a_) in enumerate(per_rank)],
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": "libnvllm_host engine C ABI: nvllm_engine_begin_step + "
                        "nvllm_engine_attention_submit / _collect (host rows, two pipeline "
                        "slots)"},
        "gpu_launches": launches,
        "clocks": clocks_all,
        "clocks_by_region": {"device": clocks_dev, "sustained": clocks_sus, "e2e": clocks_e2e},
        "sustained": {"steps": sus_steps, "ms_per_step": sus_max / sus_steps * 1e3,
                      "value": n * sus_steps * world / sus_max, "gpu_launches": launches_sus,
                      "note": "the same step back to back for >= 1.5 s after the device and "
                              "end-to-end legs; its clock record is clocks_by_region.sustained"},
        "parity": parity,
    }
    if extra:
        line["extra"] = extra
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.oracle import reference_available
        try:
            if reference_available():
                r = reference_time(spec, steps=50, warmup=1, budget_s=12.0)
                line["cpu_baseline"] = {
                    "value": r["tokens_per_s"], "unit": UNIT, "cores": r["threads"],
                    "kind": "reference",
                    "sample": f"{r['steps']} calls of the full {r['num_seqs']}-sequence batch "
                              f"(~12 s of CPU work); KV {r['kv_gbs']:.1f} GB/s"}
            else:
                line["cpu_baseline"] = None
        except Exception as exc:  # reported, never fatal
            line["cpu_baseline"] = {"error": str(exc)}
    del db, ka, va  # views of the engine's arenas
    eng.close()
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def mixed_leg(args, nvllm, lay, ka, va, dev, stream, ranks: Ranks, sampler, rank: int) -> dict:
    """The mixed prefill + decode super-batch (8 causal prefills U[512, 2048] +
    120 decodes with contexts U[256, 8192]) on the same arenas: the whole step
    with tensor-core and with fp32 prefill tiles, and its two parts
    alone (prefills; decodes), each timed like the main leg. Per part: the
    prefill's QK^T + PV FLOPs per second, the decode's algorithmic bytes per
    second. A sample of the step's rows is checked against the oracle."""
    import torch
    from nvllm.workload import make_batch
    spec = make_batch("mixed", seed=args.seed, rank=rank)
    gen = torch.Generator(device=dev)
    gen.manual_seed(3000 + rank)
    full = DeviceBatch(nvllm, spec, lay, ka, va, gen, dev, stream, nvllm.PRECISION_TF32)
    pre_idx = np.flatnonzero(spec.q_lens > 1)
    dec_idx = np.flatnonzero(spec.q_lens == 1)
    pre = DeviceBatch(nvllm, spec.subset(pre_idx), lay, ka, va, gen, dev, stream,
                      nvllm.PRECISION_TF32)
    dec = DeviceBatch(nvllm, spec.subset(dec_idx), lay, ka, va, gen, dev, stream,
                      nvllm.PRECISION_FP32)
    warm = max(args.warmup, 3)
    res = {"workload": "mixed prefill+decode super-batch (8 prefills U[512,2048] + 120 decodes "
                       "ctx U[256,8192]), 32 heads x hd 128, block 16, 65536-block arena",
           "rows_per_step": spec.n_tokens}
    legs = (("step_tf32", lambda i: full.step(nvllm.PRECISION_TF32)),
            ("step_fp32", lambda i: full.step(nvllm.PRECISION_FP32)),
            ("prefill_tf32", lambda i: pre.step(nvllm.PRECISION_TF32)),
            ("prefill_fp32", lambda i: pre.step(nvllm.PRECISION_FP32)),
            ("decode", lambda i: dec.step()))
    flops = spec.prefill_flops()
    dec_bytes = spec.subset(dec_idx).decode_algorithmic_bytes()
    for name, fn in legs:
        t, _, clk = timed_leg(fn, args.steps, warm, stream, ranks, sampler)
        ms = t / args.steps * 1e3
        r = {"ms_per_step": ms, "clocks": clk}
        if name.startswith("step"):
            r["tokens_per_s"] = spec.n_tokens / (ms / 1e3)
        if name.startswith("prefill"):
            r["tflops"] = flops / (ms / 1e3) / 1e12
        if name == "decode":
            r["hbm_gbs"] = dec_bytes / (ms / 1e3) / 1e9
        res[name] = r
    res["prefill_flops_per_step"] = flops
    res["decode_algorithmic_bytes_per_step"] = dec_bytes
    status = nvllm.get_last_error(stream)
    if status != nvllm.OK:
        raise RuntimeError(f"mixed leg: device status {nvllm.status_string(status)}")
    res["gpu_launches"] = args.steps * (2 * full.launches() + 2 * pre.launches() + dec.launches())
    if not args.no_parity:
        full.step(nvllm.PRECISION_TF32)
        torch.cuda.synchronize(dev)
        sample = list(pre_idx[:2]) + list(dec_idx[::15])
        p = oracle_parity(full, sample)
        p["max_abs"] = ranks.max(p["max_abs"])
        res["parity"] = {**p, "tol": 1e-3, "ok": p["max_abs"] <= 1e-3,
                         "precision": "tf32 prefill tiles"}
    del full, pre, dec
    torch.cuda.empty_cache()
    return res


def headsplit_leg(args, nvllm, dev, stream, ranks: Ranks, sampler, rank: int,
                  world: int) -> dict:
    """The long-context decode batch (4 sequences x 32768 positions) with its
    32 heads split over the ranks (strong scaling): rank r holds heads
    [r*H/N, (r+1)*H/N) in its own arena and runs
    nvllm_paged_attention_head_split, whose merge epilogue stores every row
    into all ranks' output buffers over NVLink; the NCCL variant (local
    attention + all_gather_into_tensor) is timed beside it. With one GPU the
    step is the plain attention call over all heads."""
    import torch
    from nvllm.workload import make_batch
    spec = make_batch("longctx", seed=args.seed)
    H, hd = spec.num_heads, spec.head_dim
    Hl = H // world
    lay = nvllm.KVLayout(spec.num_blocks, 1, spec.block_size, Hl, hd)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + rank)
    ka = torch.empty(lay.arena_shape(), device=dev).normal_(generator=gen)
    va = torch.empty_like(ka).normal_(generator=gen)
    db = DeviceBatch(nvllm, spec, lay, ka, va, gen, dev, stream, nvllm.PRECISION_FP32)
    warm = max(args.warmup, 3)
    res = {"workload": "long-context decode (4 seqs x 32768 ctx), heads split over the GPUs",
           "heads_per_gpu": Hl, "scaling": "strong"}
    per_gpu_bytes = spec.kv_bytes() / world
    if world == 1:
        t, _, clk = timed_leg(lambda i: db.step(), args.steps, warm, stream, ranks, sampler)
        res["fused"] = {"ms_per_step": t / args.steps * 1e3, "clocks": clk}
        res["gpu_launches"] = db.launches() * args.steps
        # one rank's share of an N-way split on this GPU (its heads' KV write +
        # attention, no exchange): the floor of the split's step time at N
        shares = {}
        for n in (2, 4, 8):
            sl = nvllm.KVLayout(spec.num_blocks, 1, spec.block_size, H // n, hd)
            cols = (H // n) * hd
            shape = (spec.num_blocks, 1, spec.block_size, cols)
            ks = ka.view(-1, H * hd)[:, :cols].contiguous().view(shape)
            vs = va.view(-1, H * hd)[:, :cols].contiguous().view(shape)
            part = DeviceBatch(nvllm, spec, sl, ks, vs, gen, dev, stream, nvllm.PRECISION_FP32)
            tn, _, _ = timed_leg(lambda i: part.step(), args.steps, warm, stream, ranks,
                                 sampler)
            shares[str(n)] = {"heads": H // n, "ms_per_step": tn / args.steps * 1e3,
                              "hbm_gbs": spec.kv_bytes() / n / (tn / args.steps) / 1e9}
            del part, ks, vs
        res["one_rank_share_alone"] = shares
    else:
        from nvllm.headsplit import HeadSplitGroup
        dist = ranks.dist
        grp = HeadSplitGroup(dist, n_rows=spec.n_tokens, local_cols=Hl * hd, device=dev)
        gathered = torch.empty((world, spec.n_tokens, Hl * hd), device=dev)

        def fused(i):
            db.write()
            grp.attention(db.q, ka, va, db.bt, db.cu, db.ctx, db.max_ctx, 0, lay,
                          workspace=db.ws, stream=stream)

        def nccl(i):
            db.step()
            dist.all_gather_into_tensor(gathered, db.out)

        t, _, clk = timed_leg(fused, args.steps, warm, stream, ranks, sampler)
        res["fused"] = {"ms_per_step": t / args.steps * 1e3, "clocks": clk,
                        "how": "merge epilogue stores rows into every rank's buffer over "
                               "NVLink (peer stores), bounded flag wait"}
        st = nvllm.get_last_error(stream)
        t2, _, clk2 = timed_leg(nccl, args.steps, warm, stream, ranks, sampler)
        res["nccl_allgather"] = {"ms_per_step": t2 / args.steps * 1e3, "clocks": clk2}
        res["gpu_launches"] = args.steps * (db.launches() + 2 + db.launches())
        torch.cuda.synchronize(dev)
        grp.close(dist)
        if st != nvllm.OK:
            raise RuntimeError(f"head split: device status {nvllm.status_string(st)}")
    ms = res["fused"]["ms_per_step"]
    res["tokens_per_s"] = spec.n_tokens / (ms / 1e3)
    res["hbm_gbs_per_gpu"] = per_gpu_bytes / (ms / 1e3) / 1e9
    res["kv_bytes_per_gpu"] = per_gpu_bytes
    del db, ka, va
    torch.cuda.empty_cache()
    return res


def headsplit_main(args, spec):
    """One decode batch split by heads over the ranks (strong scaling): each
    step writes the new tokens' K/V of this rank's heads and runs
    nvllm_paged_attention_head_split, whose merge epilogue stores every row into
    all ranks' output buffers over NVLink. The NCCL variant (local attention +
    all_gather_into_tensor) is timed beside it as the baseline."""
    import datetime

    import torch
    import torch.distributed as dist

    import nvllm
    from nvllm.headsplit import HeadSplitGroup

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl" if world > 1 else "gloo",
                            timeout=datetime.timedelta(seconds=120),
                            **({"device_id": dev} if world > 1 else
                               {"init_method": "tcp://127.0.0.1:29555", "rank": 0,
                                "world_size": 1}))
    nvllm.lib()
    H, hd = spec.num_heads, spec.head_dim
    assert H % world == 0, "heads must divide over the ranks"
    Hl = H // world
    lay = nvllm.KVLayout(spec.num_blocks, 1, spec.block_size, Hl, hd)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + rank)
    ka = torch.empty(lay.arena_shape(), device=dev).normal_(generator=gen)
    va = torch.empty_like(ka).normal_(generator=gen)
    n = spec.n_tokens
    q = torch.randn((n, Hl * hd), generator=gen, device=dev)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    bt = torch.from_numpy(spec.block_tables).to(dev)
    cu = torch.from_numpy(spec.cu_seqlens_q).to(dev)
    ctx = torch.from_numpy(spec.ctx_lens).to(dev)
    slots = torch.from_numpy(spec.slot_mapping()).to(dev)
    max_ctx = int(spec.ctx_lens.max())
    ws = nvllm.alloc_workspace(spec.num_seqs, 1, max_ctx, lay, device=dev)
    stream = torch.cuda.current_stream(dev)
    grp = HeadSplitGroup(dist, n_rows=n, local_cols=Hl * hd, device=dev)
    local_out = torch.empty_like(q)
    gathered = torch.empty((world, n, Hl * hd), device=dev)

    def fused_step():
        nvllm.reshape_and_cache(k, v, ka, va, slots, 0, lay, stream=stream)
        grp.attention(q, ka, va, bt, cu, ctx, max_ctx, 0, lay, workspace=ws, stream=stream)

    def nccl_step():
        nvllm.reshape_and_cache(k, v, ka, va, slots, 0, lay, stream=stream)
        nvllm.paged_attention(local_out, q, ka, va, bt, cu, ctx, 1, max_ctx, 0, lay,
                              workspace=ws, stream=stream)
        dist.all_gather_into_tensor(gathered, local_out)

    def timed(fn) -> float:
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(args.steps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        t = torch.tensor([a.elapsed_time(b) / 1e3], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(smi_device_id(local)).start()
    t_fused = timed(fused_step)
    st = nvllm.get_last_error(stream)
    t_nccl = timed(nccl_step) if world > 1 else None
    clocks = sampler.stop()
    if st != nvllm.OK:
        raise RuntimeError(f"device status {nvllm.status_string(st)}")
    tokens = n * args.steps
    value = tokens / t_fused
    per_rank_bytes = spec.kv_bytes() / world
    achieved = per_rank_bytes / (t_fused / args.steps) / 1e9
    peak = measured_peaks().get("hbm_gbs") or FALLBACK_HBM_GBS
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_fused / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic",
        "config": {**workload_config(spec), "parallelism": f"head-split x{world}",
                   "heads_per_rank": Hl},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "per": "GPU (KV bytes of its heads / step time)"},
        "nccl_allgather_baseline_ms_per_step": (t_nccl / args.steps * 1e3) if t_nccl else None,
        "gpu_launches": 5 * args.steps,
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(line))
    grp.close(dist)
    dist.barrier()
    dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# serving: the reference's engine loop (scheduler + forward_batch) end to end

SERVE_WORKLOADS = ("serve", "serve_toy", "serve_toy_seeded", "serve_router")
SERVE_METRIC = "e2e serving output tokens/s (continuous batching, greedy)"
SERVE_DEFAULT_STEPS = {"serve": 3, "serve_toy": 10, "serve_toy_seeded": 10, "serve_router": 2}


def model_flops(model: dict, tokens_computed: int, rows_sampled: int) -> float:
    """Projection FLOPs of forward_batch: 2 * (4 d^2 + 2 d ffn) per layer per
    flattened token, plus the LM head (2 d vocab) per sampled row."""
    d, f, v, L = model["hidden"], model["ffn"], model["vocab"], model["layers"]
    return 2.0 * L * (4 * d * d + 2 * d * f) * tokens_computed + 2.0 * d * v * rows_sampled


def reference_serve(spec, budget_s: float = 20.0) -> dict:
    """The reference's own engine loop (ContinuousScheduler + forward_batch with
    its real matmuls, oracle/_ref) on the host cores. The toy workloads run
    whole; for the 4096-wide model the sample is the workload's first requests
    with completions capped at 8 tokens, as many as fit the time budget."""
    from oracle.oracle import RefPath
    ref = RefPath()
    threads = os.cpu_count() or 1
    if spec.name != "serve":
        steps, secs = ref.generate_timed(spec.model, spec.num_blocks, spec.block_size,
                                         spec.max_batch, spec.max_tokens_per_step, spec.watermark,
                                         spec.prompts, spec.max_new)
        return {"tokens": spec.output_tokens, "seconds": secs, "steps": steps, "threads": threads,
                "sample": f"the whole workload ({len(spec.prompts)} requests, "
                          f"{spec.output_tokens} output tokens)"}
    cap = 8
    n = 1
    prompts, max_new = spec.prompts[:n], [min(m, cap) for m in spec.max_new[:n]]
    steps, secs = ref.generate_timed(spec.model, 2 * spec.engine_limits()["max_blocks_per_seq"] + 8,
                                     spec.block_size, spec.max_batch, spec.max_tokens_per_step, 0,
                                     prompts, max_new)
    return {"tokens": int(sum(max_new)), "seconds": secs, "steps": steps, "threads": threads,
            "sample": f"first {n} request(s) of the workload ({sum(len(p) for p in prompts)} prompt "
                      f"tokens), completions capped at {cap} tokens; scheduling loop only "
                      f"(model construction excluded)"}


def reference_serve_main(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from nvllm.serving import make_serve, serve_config
    from oracle.oracle import reference_available
    spec = make_serve(args.workload, seed=args.seed)
    if not reference_available():
        print(json.dumps({"impl": "reference", "metric": SERVE_METRIC,
                          "unavailable": "oracle/_ref (the reference's C++ built from its sources) "
                                         "is not present on this machine"}))
        return 0
    runs = []
    for _ in range(args.steps if spec.name != "serve" else 1):
        runs.append(reference_serve(spec))
    tok = sum(r["tokens"] for r in runs)
    secs = sum(r["seconds"] for r in runs)
    value = tok / secs
    line = {
        "impl": "reference", "metric": SERVE_METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": len(runs), "warmup": 0,
        "ms_per_step": secs / len(runs) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "config": serve_config(spec),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": runs[0]["threads"],
                         "kind": "reference", "sample": runs[0]["sample"]},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def serve_main(args):
    """K complete serving runs of the workload's requests (one run = one step)
    per GPU: the generator schedules, uploads each iteration's metadata and
    token ids from pinned host memory, runs forward_batch on the device and
    reads the sampled ids back, until every request has finished. Under
    torchrun every rank serves its own requests (sequence partitioning)."""
    # The host library is loaded before torch so that its cuBLAS references bind
    # to the CUDA toolkit's cuBLAS it was linked against (which has the bf16x9
    # mode) rather than to the copy torch brings.
    from nvllm.host import GEMM_BF16X9, GEMM_FP32, GEMM_TF32X3, Engine, Generator, Model, host_lib
    host_lib()
    import torch
    import nvllm
    from nvllm.serving import make_serve, serve_config

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    nvllm.lib()
    spec = make_serve(args.workload, seed=args.seed + (rank if args.workload == "serve" else 0))
    lay = nvllm.KVLayout(spec.num_blocks, spec.model["layers"], spec.block_size,
                         spec.model["heads"], spec.model["head_dim"])
    eng = Engine(lay, device=local, **spec.engine_limits())
    gemm = {"fp32": GEMM_FP32, "bf16x9": GEMM_BF16X9, "tf32x3": GEMM_TF32X3}[args.gemm]
    model = Model(spec.model, eng, gemm_math=gemm, graph_max_tokens=args.graph_max_tokens)
    precision = nvllm.PRECISION_TF32 if args.precision == "tf32" else nvllm.PRECISION_FP32
    estream = torch.cuda.ExternalStream(eng.stream(), device=dev)

    def one_run():
        gen = Generator(eng, model, spec.max_batch, spec.max_tokens_per_step, spec.watermark,
                        precision=precision)
        for i, (p, m) in enumerate(zip(spec.prompts, spec.max_new)):
            gen.add_request(i + 1, p, m)
        gen.run()
        m = gen.metrics()
        gen.close()
        return m

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(smi_device_id(local)).start()
    for _ in range(args.warmup):
        one_run()
    torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(estream)
    ms = [one_run() for _ in range(args.steps)]
    e1.record(estream)
    torch.cuda.synchronize(dev)
    barrier()
    elapsed = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    clocks = sampler.stop()
    status = nvllm.get_last_error(eng.stream())
    if status != nvllm.OK:
        raise RuntimeError(f"device status {nvllm.status_string(status)}")
    model.close()
    eng.close()

    out_tokens = sum(m.total_tokens_generated for m in ms)
    assert out_tokens == spec.output_tokens * args.steps
    computed = sum(m.total_tokens_computed for m in ms)
    iters = sum(m.total_iterations for m in ms)
    value = out_tokens * world / elapsed
    flops = model_flops(spec.model, computed, out_tokens)
    peaks = measured_peaks()
    peak = peaks.get("bf16_tflops")
    peak_src = "measured (dense bf16, burst)" if peak else "fallback"
    if not peak:
        peak = 1590.0
    achieved = flops / elapsed / 1e12
    h2d = sum(m.h2d_bytes for m in ms) // args.steps
    d2h = sum(m.d2h_bytes for m in ms) // args.steps
    line = {
        "metric": SERVE_METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded prompts; LCG weights of the reference model)",
        "config": {**serve_config(spec), "gemm": args.gemm, "prefill_precision": args.precision,
                   "graph_max_tokens": args.graph_max_tokens,
                   "parallelism": f"sequence-partitioned x{world}",
                   "engine_iterations_per_step": iters / args.steps,
                   "tokens_computed_per_step": computed / args.steps,
                   "l2": "weights (>= 1.5 MB toy, 3.4 GB wide) and KV stream every iteration; "
                         "no flush"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "kernel": "whole engine iteration (fp32 projections dominate)",
                     "algorithmic_flops_per_step": flops / args.steps,
                     "note": "projection FLOPs over the timed region; the GEMMs run in fp32 "
                             "(FFMA, or bf16x9 emulation) against the dense bf16 peak",
                     "traffic": None},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": "libnvllm_host generator C ABI (nvllm_generator_add_request + "
                        "nvllm_generator_run): every engine iteration uploads its metadata and "
                        "token ids from pinned host memory and reads the sampled ids back, so "
                        "the timed value is itself end to end"},
        "gpu_launches": sum(m.kernel_launches for m in ms),
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle.oracle import reference_available
        try:
            if reference_available():
                r = reference_serve(spec)
                line["cpu_baseline"] = {"value": r["tokens"] / r["seconds"], "unit": UNIT,
                                        "cores": r["threads"], "kind": "reference",
                                        "sample": r["sample"]}
            else:
                line["cpu_baseline"] = None
        except Exception as exc:  # reported, never fatal
            line["cpu_baseline"] = {"error": str(exc)}
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def serve_router_main(args):
    """Config-5 serving over the GPUs of one box through nvllm_router: one
    stream of 128 x N requests (lognormal prompts, 16 / 512 completions) placed
    by the router on the GPU with the least outstanding work; every GPU has its
    own engine (arena, allocator), model, scheduler and engine thread, and
    nothing is shared on the data path. One process drives the N devices (the
    engine threads are C++); under torchrun rank 0 does and the other ranks
    return. One step = one complete run of the stream; its time is taken on
    every device with CUDA events on that device's engine stream (from before
    the first request is placed to after the router went idle), max over the
    devices."""
    from nvllm.host import GEMM_TF32X3, Engine, Generator, Model, Router, host_lib
    host_lib()
    import torch
    import nvllm
    from nvllm.serving import make_serve, serve_config

    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    n_gpu = args.gpus
    if torch.cuda.device_count() < n_gpu:
        raise RuntimeError(f"{n_gpu} GPUs asked for, {torch.cuda.device_count()} visible")
    nvllm.lib()
    spec = make_serve("serve", seed=args.seed, requests=128 * n_gpu)
    need = sum((len(p_) + m_ + spec.block_size - 1) // spec.block_size
               for p_, m_ in zip(spec.prompts, spec.max_new))
    blocks = int(need * 1.25 / n_gpu) + 256  # a GPU's share with room for imbalance
    lay = nvllm.KVLayout(blocks, spec.model["layers"], spec.block_size, spec.model["heads"],
                         spec.model["head_dim"])
    limits = spec.engine_limits()
    precision = nvllm.PRECISION_TF32 if args.precision == "tf32" else nvllm.PRECISION_FP32
    lanes = []
    for d in range(n_gpu):
        torch.cuda.set_device(d)
        eng = Engine(lay, device=d, **limits)
        model = Model(spec.model, eng, gemm_math=GEMM_TF32X3,
                      graph_max_tokens=args.graph_max_tokens)
        gen = Generator(eng, model, spec.max_batch, spec.max_tokens_per_step, spec.watermark,
                        precision=precision)
        lanes.append((eng, model, gen))
    torch.cuda.set_device(0)
    router = Router([g for _, _, g in lanes])
    streams = [torch.cuda.ExternalStream(e.stream(), device=torch.device("cuda", d))
               for d, (e, _, _) in enumerate(lanes)]
    samplers = [ClockSampler(smi_device_id(d)).start() for d in range(n_gpu)]

    def one_run(run: int):
        # the stream arrives as one burst: placed in one call, each GPU woken
        # once with its whole share
        base = (run + 1) * 1_000_000
        router.add_requests([base + i for i in range(len(spec.prompts))], spec.prompts,
                            spec.max_new)
        router.wait_idle()

    for r in range(args.warmup):
        one_run(r)
    for d in range(n_gpu):
        torch.cuda.synchronize(d)
    before = [router.metrics(d) for d in range(n_gpu)]
    placed0 = [router.placed(d) for d in range(n_gpu)]
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n_gpu)]
    t0 = time.monotonic()
    for d in range(n_gpu):
        with torch.cuda.device(d):
            ev[d][0].record(streams[d])
    for r in range(args.steps):
        one_run(args.warmup + r)
    for d in range(n_gpu):
        with torch.cuda.device(d):
            ev[d][1].record(streams[d])
    for d in range(n_gpu):
        torch.cuda.synchronize(d)
    t1 = time.monotonic()
    per_dev = [ev[d][0].elapsed_time(ev[d][1]) / 1e3 for d in range(n_gpu)]
    elapsed = max(per_dev)
    clocks = [samplers[d].window(t0, t1) for d in range(n_gpu)]
    for smp in samplers:
        smp.stop()
    after = [router.metrics(d) for d in range(n_gpu)]
    for _, _, gen in lanes:
        st = nvllm.get_last_error(gen.engine.stream())
        if st != nvllm.OK:
            raise RuntimeError(f"device status {nvllm.status_string(st)}")
    gen_tok = [a.total_tokens_generated - b.total_tokens_generated for a, b in zip(after, before)]
    out_tokens = sum(gen_tok)
    assert out_tokens == spec.output_tokens * args.steps, (out_tokens, spec.output_tokens)
    computed = sum(a.total_tokens_computed - b.total_tokens_computed
                   for a, b in zip(after, before))
    placed = [router.placed(d) - placed0[d] for d in range(n_gpu)]
    value = out_tokens / elapsed
    flops = model_flops(spec.model, computed, out_tokens)
    peak = measured_peaks().get("bf16_tflops") or 1590.0
    h2d = sum(a.h2d_bytes - b.h2d_bytes for a, b in zip(after, before)) // args.steps
    d2h = sum(a.d2h_bytes - b.d2h_bytes for a, b in zip(after, before)) // args.steps
    reasons = sorted({x for c in clocks for x in c["reasons"]})
    sm = [c["sm_mhz"] for c in clocks if c["sm_mhz"]]
    line = {
        "metric": SERVE_METRIC, "value": value, "unit": UNIT, "n_gpus": n_gpu,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded prompts; LCG weights of the reference model)",
        "config": {**serve_config(spec), "workload": "e2e serving, 4096-wide 4-layer model, "
                   "one stream of 128 requests per GPU through the router"},
        "parallelism": f"sequence-partitioned x{n_gpu} (router: least outstanding work)",
        "gemm": "tf32x3", "prefill_precision": args.precision,
        "graph_max_tokens": args.graph_max_tokens,
        "per_gpu": [{"gpu": d, "requests": placed[d], "tokens_generated": gen_tok[d],
                     "seconds": per_dev[d] / args.steps} for d in range(n_gpu)],
        "roofline": {"bound": "tensor", "achieved": flops / elapsed / 1e12 / n_gpu,
                     "peak": peak, "unit": "TFLOP/s", "frac": flops / elapsed / 1e12 / n_gpu / peak,
                     "per": "GPU", "kernel": "whole engine iteration (fp32 projections dominate)",
                     "traffic": None},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": "libnvllm_host router C ABI (nvllm_router_add_request + "
                        "nvllm_router_wait_idle); every engine iteration uploads its metadata "
                        "and token ids and reads the sampled ids back"},
        "gpu_launches": sum(a.kernel_launches - b.kernel_launches for a, b in zip(after, before)),
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None,
                   "sm_max_mhz": max((c["sm_max_mhz"] or 0) for c in clocks) or None,
                   "reasons": reasons, "samples": sum(c["samples"] for c in clocks),
                   "per_gpu": clocks},
    }
    router.close()
    for eng, model, gen in lanes:
        gen.close()
        model.close()
        eng.close()
    print(json.dumps(line))
    return 0


HEADMODEL_METRIC = "long-context decode tokens/s in the model (heads split over the GPUs)"


def headmodel_main(args):
    """Long-context decode inside the 4096-wide model with its heads split over
    the ranks (nvllm_model head_ranks = N): 4 requests of 32768 prompt tokens
    are prefilled through the generator (not timed), then `steps` decode
    iterations (4 new tokens each, every rank computing the same tokens) are
    timed with CUDA events on the engine's stream, max over ranks. Strong
    scaling: the work per step is fixed, each rank streams heads / N of the KV
    and a 1 / N slice of W_q, W_k, W_v; W_o, the FFN and the LM head are
    replicated."""
    from nvllm.host import GEMM_TF32X3, Engine, Generator, Model, host_lib
    host_lib()
    import torch
    import nvllm
    from nvllm.headsplit import ModelHeads
    from nvllm.serving import make_serve, serve_config

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    nvllm.lib()
    spec = make_serve("longctx_model", seed=args.seed)
    m = spec.model
    lay = nvllm.KVLayout(spec.num_blocks, m["layers"], spec.block_size, m["heads"] // world,
                         m["head_dim"])
    limits = spec.engine_limits()
    eng = Engine(lay, device=local, **limits)
    model = Model(m, eng, gemm_math=GEMM_TF32X3, head_ranks=world)
    heads = None
    if world > 1:
        heads = ModelHeads(dist, limits["max_tokens"], m["hidden"], dev)
        heads.attach(model)
    precision = nvllm.PRECISION_TF32 if args.precision == "tf32" else nvllm.PRECISION_FP32
    gen = Generator(eng, model, spec.max_batch, spec.max_tokens_per_step, spec.watermark,
                    precision=precision)
    for i, (p_, n_) in enumerate(zip(spec.prompts, spec.max_new)):
        gen.add_request(i + 1, p_, n_)
    estream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    n_seq = len(spec.prompts)
    # prefill (a whole prompt per iteration), until an iteration is pure decode
    for _ in range(2 * n_seq + 4):
        s = gen.step()
        if s["scheduled_tokens"] == n_seq and s["batch_size"] == n_seq:
            break
    else:
        raise RuntimeError("the prompts were not all prefilled within the expected iterations")
    for _ in range(args.warmup):
        gen.step()
    m0 = gen.metrics()

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(smi_device_id(local)).start()
    torch.cuda.synchronize(dev)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(estream)
    for _ in range(args.steps):
        gen.step()
    e1.record(estream)
    torch.cuda.synchronize(dev)
    barrier()
    elapsed = max_over_ranks(e0.elapsed_time(e1) / 1e3)
    clocks = sampler.stop()
    m1 = gen.metrics()
    status = nvllm.get_last_error(eng.stream())
    if status != nvllm.OK:
        raise RuntimeError(f"device status {nvllm.status_string(status)}")
    tokens = m1.total_tokens_generated - m0.total_tokens_generated
    assert tokens == n_seq * args.steps, tokens
    # bytes a rank streams per decode iteration: its heads' KV of every layer
    # (the context grows by one token a step) and the weights it reads
    D, F, V, Lyr = m["hidden"], m["ffn"], m["vocab"], m["layers"]
    ctx = len(spec.prompts[0]) + args.warmup + args.steps // 2
    kv = n_seq * ctx * Lyr * 2 * (D // world) * 4
    w = Lyr * (3 * D * (D // world) + D * D + 2 * D * F) * 4 + D * V * 4
    per_step = elapsed / args.steps
    hbm = measured_peaks().get("hbm_gbs") or 6650.0
    achieved = (kv + w) / per_step / 1e9
    line = {
        "metric": HEADMODEL_METRIC, "value": tokens / elapsed, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded prompts; LCG weights of the reference model)",
        "config": {**serve_config(spec), "gemm": "tf32x3", "prefill_precision": args.precision,
                   "parallelism": f"heads split x{world}" if world > 1 else "one GPU",
                   "context_tokens": ctx,
                   "l2": "KV and weights (>= 7 GB a step) far above L2; no flush"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": "measured (copy)",
                     "kernel": "whole decode iteration (KV of this rank's heads + weights)",
                     "kv_bytes_per_step": kv, "weight_bytes_per_step": w, "traffic": None},
        "e2e": {"value": tokens / elapsed, "unit": UNIT,
                "h2d_bytes_per_step": (m1.h2d_bytes - m0.h2d_bytes) // args.steps,
                "d2h_bytes_per_step": (m1.d2h_bytes - m0.d2h_bytes) // args.steps,
                "path": "libnvllm_host generator C ABI (nvllm_generator_step): metadata and "
                        "token ids up, sampled ids down every iteration"},
        "gpu_launches": m1.kernel_launches - m0.kernel_launches,
        "clocks": clocks,
    }
    if rank == 0 and world == 1:
        line["cpu_baseline"] = {
            "value": None, "unit": UNIT, "cores": os.cpu_count(), "kind": "reference",
            "sample": "not timed: the reference's CPU path needs about an hour to prefill "
                      "4 x 32768 tokens of this model (29 prefill tok/s measured on the "
                      "4096-wide model); its attention alone at this shape is the longctx "
                      "workload's cpu_baseline"}
    gen.close()
    torch.cuda.synchronize(dev)
    if heads is not None:
        barrier()
        heads.close(dist)
    model.close()
    eng.close()
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# the model's projection GEMMs (profiling sweeps; tables on stderr)

GEMM_SHAPES = [(m, k, n) for m in (26, 128) for (k, n) in ((4096, 12288), (4096, 4096), (4096, 11008),
                                                        (11008, 4096), (4096, 32000))] + \
          [(m, k, n) for m in (512, 4096) for (k, n) in ((4096, 12288), (4096, 11008),
                                                         (11008, 4096))]


def gemm_main(args) -> int:
    """--workload gemm: nvllm_gemm_tf32x3 against cuBLAS fp32 (torch.matmul,
    TF32 off) on the projection shapes of the 4096-wide model, decode-size and
    prefill-size. Per shape: time per call (CUDA events, after warm-up) with the
    weights pre-split into hi / lo (the model's layout) and split on chip, the
    cuBLAS time, and the error of both against a float64 product. --once m,k,n
    runs a single pre-split call of one shape (for a profiler)."""
    import ctypes

    import torch

    import nvllm
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

    shapes = GEMM_SHAPES if not args.shapes else [tuple(int(v) for v in s.split(",")) for s in args.shapes]
    log(f"{'m':>6} {'k':>6} {'n':>6}  {'presplit us':>11} {'TFLOP/s':>8} {'onchip us':>10} "
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
        log(f"{m:6d} {k:6d} {n:6d}  {times['pre']:11.1f} {fl / times['pre'] / 1e6:8.1f} "
              f"{times['chip']:10.1f} {times['cublas']:10.1f} {fl / times['cublas'] / 1e6:8.1f} "
              f"{times['cublas'] / times['pre']:8.2f} {err_pre:12.1e} {err_cb:10.1e}")
    assert nvllm.get_last_error(torch.cuda.current_stream().cuda_stream) == nvllm.OK
    return 0


GEMM_SKINNY_SHAPES = [(m, k, n, b) for m in (1, 8, 16, 26, 32, 48, 64, 96, 128)
          for (k, n, b) in ((4096, 4096, 3), (4096, 4096, 1), (4096, 11008, 1), (11008, 4096, 1),
                            (4096, 32000, 1))]


def gemm_skinny_main(args) -> int:
    """--workload gemm_skinny: nvllm_gemm_skinny (FFMA, decode-size rows, batch
    weight matrices per call) and nvllm_gemm_decode_tc (tcgen05, m <= 32) against
    cuBLAS and the tcgen05 GEMM on the same shapes, with the weight stream's
    bandwidth; x cuBLAS is for the faster of the first two. --once m,k,n,batch
    runs a single call of one shape (for a profiler)."""
    import ctypes

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

    if args.once:
        m, k, n, b = (int(v) for v in args.once.split(","))
        x, w, outs, ws = setup(m, k, n, b)
        skinny(x, w, outs, ws, m, k, n, b, fn=L.nvllm_gemm_decode_tc if m <= 32 else L.nvllm_gemm_skinny)
        torch.cuda.synchronize()
        return 0

    shapes = GEMM_SKINNY_SHAPES if not args.shapes else [tuple(int(v) for v in s.split(",")) for s in args.shapes]
    log(f"{'m':>4} {'k':>6} {'n':>6} {'b':>2}  {'skinny us':>9} {'GB/s':>7} {'TFLOP/s':>7} "
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
        log(f"{m:4d} {k:6d} {n:6d} {b:2d}  {us:9.1f} {b * k * n * 4 / us / 1e3:7.0f} "
              f"{2.0 * m * k * n * b / us / 1e6:7.1f} {ud:9.1f} {b * k * n * 4 / ud / 1e3:7.0f} "
              f"{times['cublas']:9.1f} {times['tc']:9.1f} {times['cublas'] / best:8.2f} "
              f"{err_sk:8.1e} {err_tc:8.1e}")
    assert nvllm.get_last_error(torch.cuda.current_stream().cuda_stream) == nvllm.OK
    return 0



def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 1000 attention calls; 3 or 10 serving runs)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["nvllm", "reference"], default="nvllm")
    ap.add_argument("--workload", choices=["decode", "mixed", "longctx", "decode_small",
                                           "mixed_small", "longctx_model", "gemm", "gemm_skinny",
                                           *SERVE_WORKLOADS],
                    default="decode")
    ap.add_argument("--gemm", choices=["fp32", "bf16x9", "tf32x3"], default=None,
                    help="projection arithmetic of the serving workloads: cuBLAS FFMA, cuBLAS "
                         "bf16x9, or this library's GEMMs (tcgen05 3xTF32 above 32 rows and at "
                         "17-32, FFMA at <= 16); default tf32x3 for serve, fp32 for the toy "
                         "model (whose 128-wide projections give the tensor-core GEMMs one to "
                         "three tiles)")
    ap.add_argument("--graph-max-tokens", type=int, default=None,
                    help="serving: engine iterations of at most this many new tokens replay a "
                         "CUDA graph per padded bucket (0: eager; default 512, or 0 for serve "
                         "with cuBLAS projections, which run slower on padded shapes than the "
                         "launches a graph saves)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--precision", choices=["fp32", "tf32"], default=None,
                    help="prefill tile arithmetic (decode is always fp32): fp32 FFMA, or tcgen05 "
                         "with two-term bf16 products (1e-3); default tf32 for a serving workload whose "
                         "projections run on the tcgen05 GEMMs, else fp32")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="decode workload: skip the mixed and head-split legs of `extra`")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the oracle check of the timed batch after the timed regions")
    ap.add_argument("--head-split", action="store_true",
                    help="split the batch's heads over the ranks (long-context decode)")
    ap.add_argument("--head-slice", type=int, default=1,
                    help="attention workloads: keep 1/N of the heads (one rank's share of an "
                         "N-way head split, run alone on one GPU)")
    ap.add_argument("--shapes", nargs="*", default=None,
                    help="gemm workloads: m,k,n (gemm) or m,k,n,batch (gemm_skinny) per shape")
    ap.add_argument("--reps", type=int, default=10, help="gemm workloads: timed calls per shape")
    ap.add_argument("--once", default=None,
                    help="gemm workloads: one call of one shape, for a profiler")
    args = ap.parse_args()
    if args.workload == "gemm":
        return gemm_main(args)
    if args.workload == "gemm_skinny":
        return gemm_skinny_main(args)
    if args.warmup < 3:
        log("warm-up raised to 3 steps")
        args.warmup = 3
    if args.workload == "longctx_model":
        if args.steps is None:
            args.steps = 32
        if args.precision is None:
            args.precision = "tf32"
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "the reference's CPU path needs about an hour to prefill "
                                  "4 x 32768 tokens of the 4096-wide model"}))
            return 0
        return headmodel_main(args)
    if args.workload in SERVE_WORKLOADS:
        if args.steps is None:
            args.steps = SERVE_DEFAULT_STEPS[args.workload]
        if args.gemm is None:
            args.gemm = "tf32x3" if args.workload in ("serve", "serve_router") else "fp32"
        if args.graph_max_tokens is None:
            args.graph_max_tokens = 0 if args.workload == "serve" and args.gemm != "tf32x3" else 512
        if args.precision is None:
            args.precision = "tf32" if args.gemm == "tf32x3" else "fp32"
        if args.workload == "serve_router":
            if args.impl == "reference":
                args.workload = "serve"
                return reference_serve_main(args)
            return serve_router_main(args)
        return reference_serve_main(args) if args.impl == "reference" else serve_main(args)
    if args.steps is None:
        args.steps = 1000
    if args.precision is None:
        args.precision = "fp32"
    from nvllm.workload import make_batch
    spec = make_batch(args.workload, seed=args.seed)
    if args.head_slice > 1:
        import dataclasses
        spec = dataclasses.replace(spec, num_heads=spec.num_heads // args.head_slice)
    if args.impl == "reference":
        return reference_main(args, spec)
    if args.head_split:
        return headsplit_main(args, spec)
    return nvllm_main(args, spec)


if __name__ == "__main__":
    sys.exit(main())
