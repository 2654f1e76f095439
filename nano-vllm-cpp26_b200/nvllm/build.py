"""Builds libnvllm.so (the sm_100a kernels + C ABI) in-tree.

    python -m nvllm.build          (from nano-vllm-cpp26_b200/)

nvcc compiles every csrc/*.cu for sm_100a with relocatable device code and
links them into lib/libnvllm.so; the static CUDA runtime is linked in so the
library depends only on the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
CSRC = PKG / "csrc"
LIB = PKG / "lib"
INCLUDE = PKG.parent / "include"
LIBNAME = "libnvllm.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++20", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise FileNotFoundError("nvcc not found")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / LIBNAME
    deps = sources() + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "nvllm.h", Path(__file__)]
    if not force and not _stale(out, deps):
        return out
    objdir = LIB / "_obj"
    objdir.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        objs.append(obj)
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, pr in procs:
        outp, _ = pr.communicate()
        if pr.returncode != 0 or (verbose and outp):
            print(outp.decode(errors="replace"))
        if pr.returncode != 0:
            failed.append(src.name)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objs),
           "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    import sys
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
