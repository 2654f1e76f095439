"""Builds the two in-tree libraries.

    python -m nvllm.build          (from nano-vllm-cpp26_b200/)

* lib/libnvllm.so: nvcc compiles every csrc/*.cu for sm_100a with relocatable
  device code and links them; the static CUDA runtime is linked in so the
  library depends only on the driver.
* lib/libnvllm_host.so: g++ -std=c++23 compiles host/*.cpp (block allocator,
  metadata packer, engine, device model, their C ABI) against libnvllm.so,
  cuBLAS (the model's fp32 projections) and the static CUDA runtime.
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
HOSTLIB = "libnvllm_host.so"
HOST = PKG / "host"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

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
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h")) + [Path(__file__)]
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


def build_host(force: bool = False, verbose: bool = False) -> Path:
    """Compiles host/*.cpp into lib/libnvllm_host.so (needs lib/libnvllm.so)."""
    core = build(force=False, verbose=verbose)
    out = LIB / HOSTLIB
    srcs = sorted(HOST.glob("*.cpp"))
    deps = srcs + sorted(HOST.glob("*.hpp")) + sorted(INCLUDE.glob("*.h")) + [core, Path(__file__)]
    if not force and not _stale(out, deps):
        return out
    cxx = shutil.which("g++") or "g++"
    tmp = out.with_suffix(".so.tmp")
    cmd = [cxx, "-std=c++23", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-pthread",
           f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}", *map(str, srcs), "-o", str(tmp),
           f"-L{LIB}", "-lnvllm", f"-L{CUDA_HOME / 'lib64'}", "-lcublas", "-lcudart_static",
           "-ldl", "-lrt",
           "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    import sys
    p = build(force="--force" in sys.argv, verbose=True)
    print(p)
    print(build_host(force="--force" in sys.argv, verbose=True))
