"""torchrun worker for the head-parallel model test (tests/test_gpu_multigpu.py).

Every rank runs the generator on the reference's 4096-wide token trace with a
head-parallel model: its engine holds heads [r*H/N, (r+1)*H/N), QKV runs for
those heads, nvllm_head_gather collects every rank's attention rows before
W_o, and the rest of the forward is replicated. Every rank must write the
reference's trace: every batch, every sampled token, the top-8 logits within
LOGIT_RTOL of the row's largest; once with cuBLAS FFMA projections and once
with this library's GEMMs.
"""
import datetime
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "nano-vllm-cpp26_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import nvllm  # noqa: E402
from nvllm.headsplit import ModelHeads  # noqa: E402
from nvllm.host import GEMM_FP32, GEMM_TF32X3, Engine, Generator, Model  # noqa: E402

from helpers import LOGIT_RTOL, load_trace, trace_requests  # noqa: E402
from oracle.oracle import read_trace  # noqa: E402


def run(rank, world, dev, gemm_math, tmpdir):
    cfg, z, steps = load_trace("tokens_wide")
    max_batch, max_tokens, watermark = (int(x) for x in z["sched"])
    H = cfg["heads"]
    lay = nvllm.KVLayout(int(z["num_blocks"]), cfg["layers"], int(z["block_size"]), H // world,
                         cfg["head_dim"])
    prompts, max_new = trace_requests(z)
    longest = max(len(p) + m for p, m in zip(prompts, max_new))
    B = int(z["block_size"])
    rows = max(max_tokens, longest)
    eng = Engine(lay, device=dev.index, max_seqs=max_batch, max_tokens=rows,
                 max_blocks_per_seq=(longest + B - 1) // B)
    model = Model(cfg, eng, scales=z["scales"][:2], gemm_math=gemm_math, head_ranks=world)
    heads = ModelHeads(dist, rows, cfg["hidden"], dev)
    heads.attach(model)
    gen = Generator(eng, model, max_batch, max_tokens, watermark)
    try:
        for i, (p, m) in enumerate(zip(prompts, max_new)):
            gen.add_request(i + 1, p, m)
        path = os.path.join(tmpdir, f"rank{rank}_gemm{gemm_math}.trace")
        gen.trace(path)
        n_steps = gen.run()
        gen.trace(None)
        assert n_steps == len(steps), (n_steps, len(steps))
        mine = read_trace(path)
        for i, (a, b) in enumerate(zip(mine, steps)):
            assert np.array_equal(a["record"], b["record"]), f"step {i}: batch"
            assert np.array_equal(a["sampled"], b["sampled"]), f"step {i}: tokens"
            scale = np.abs(b["top_val"]).max(axis=1, keepdims=True)
            assert (np.abs(a["top_val"] - b["top_val"]) <= LOGIT_RTOL * scale).all(), f"step {i}"
        m = gen.metrics()
        assert m.total_requests_completed == len(prompts)
    finally:
        gen.close()
        torch.cuda.synchronize(dev)
        dist.barrier()
        heads.close(dist)
        model.close()
        eng.close()


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    nvllm.lib()
    with tempfile.TemporaryDirectory() as tmpdir:
        for gemm_math in (GEMM_FP32, GEMM_TF32X3):
            run(rank, world, dev, gemm_math, tmpdir)
            print(f"rank {rank}: head-parallel model over {world} ranks, gemm {gemm_math} ok",
                  flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
