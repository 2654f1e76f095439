"""Multi-GPU parity: the head-split attention (rows stored into peer GPUs'
buffers by the merge epilogue) against the single-GPU full-head result, run
as a torchrun job of 2, 4 or 8 ranks (tests/mp_head_split.py), each size
skipped when the box has fewer GPUs.
NVLS is disabled in NCCL for the job (no multicast objects are involved in
the kernels themselves)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_split(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "280", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(ROOT / "tests" / "mp_head_split.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(f"head split over {world} ranks ok") == world


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_parallel_model(world):
    """The whole model with its heads split over the ranks (tests/mp_model_heads.py):
    every rank reproduces the reference's 4096-wide token trace."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", str(ROOT / "tests" / "mp_model_heads.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=420)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count(f"head-parallel model over {world} ranks") == 2 * world
