"""torchrun worker for the head-split parity test (tests/test_gpu_multigpu.py).

Every rank builds the same long-context decode batch (32 heads x hd 128,
block size 16) on its own GPU, computes the full-head reference with
nvllm_paged_attention, then computes its slice of the heads with
nvllm_paged_attention_head_split over three epochs. Each rank's gathered
output must equal the full-head result bit for bit (the per-head arithmetic
is the same), and so must the NCCL all-gather of the local outputs.
"""
import datetime
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "nano-vllm-cpp26_b200"))

import nvllm  # noqa: E402
from nvllm.headsplit import HeadSplitGroup  # noqa: E402


def main() -> int:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    nvllm.lib()
    H, hd, B = 32, 128, 16
    assert H % world == 0
    Hl = H // world
    ctx = np.array([8192, 5000, 777, 8191, 1, 256], np.int32)
    S = len(ctx)
    nbs = (ctx + B - 1) // B
    nb = int(nbs.sum()) + 16
    rng = np.random.default_rng(5)
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((S, int(nbs.max())), np.int32)
    off = 0
    for s in range(S):
        bt[s, :nbs[s]] = perm[off:off + nbs[s]]
        off += nbs[s]
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    ka_full = torch.empty((nb, 1, B, H * hd), device=dev).normal_(generator=gen)
    va_full = torch.empty_like(ka_full).normal_(generator=gen)
    q_full = torch.randn((S, H * hd), generator=gen, device=dev)
    bt_d = torch.from_numpy(bt).to(dev)
    cu = torch.arange(S + 1, dtype=torch.int32, device=dev)
    ctx_d = torch.from_numpy(ctx).to(dev)
    max_ctx = int(ctx.max())

    lay_full = nvllm.KVLayout(nb, 1, B, H, hd)
    ref = torch.empty_like(q_full)
    nvllm.paged_attention(ref, q_full, ka_full, va_full, bt_d, cu, ctx_d, 1, max_ctx, 0, lay_full)

    cols = slice(rank * Hl * hd, (rank + 1) * Hl * hd)
    ka = ka_full[..., cols].contiguous()
    va = va_full[..., cols].contiguous()
    q = q_full[:, cols].contiguous()
    del ka_full, va_full
    lay = nvllm.KVLayout(nb, 1, B, Hl, hd)
    ws = nvllm.alloc_workspace(S, 1, max_ctx, lay, device=dev)

    grp = HeadSplitGroup(dist, n_rows=S, local_cols=Hl * hd, device=dev)
    for epoch in range(3):
        out = grp.attention(q, ka, va, bt_d, cu, ctx_d, max_ctx, 0, lay, workspace=ws)
        torch.cuda.synchronize(dev)
        st = nvllm.get_last_error()
        assert st == nvllm.OK, f"rank {rank} epoch {epoch}: {nvllm.status_string(st)}"
        assert torch.equal(out, ref), (
            f"rank {rank} epoch {epoch}: max-abs {(out - ref).abs().max().item()}")

    # NCCL baseline: local heads, then all-gather and head-major interleave
    local_out = torch.empty_like(q)
    nvllm.paged_attention(local_out, q, ka, va, bt_d, cu, ctx_d, 1, max_ctx, 0, lay, workspace=ws)
    gathered = torch.empty((world, S, Hl * hd), device=dev)
    dist.all_gather_into_tensor(gathered, local_out)
    nccl_out = gathered.permute(1, 0, 2).reshape(S, H * hd)
    assert torch.equal(nccl_out, ref)

    grp.close(dist)
    dist.barrier()
    dist.destroy_process_group()
    print(f"rank {rank}: head split over {world} ranks ok (max |ref| "
          f"{ref.abs().max().item():.3f}, scale {1 / math.sqrt(hd):.4f})")
    return 0


if __name__ == "__main__":
    sys.exit(main())
