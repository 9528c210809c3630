"""Build libpageserve_b200.so in-tree with nvcc for sm_100a.

    python -m pageserve_b200.build            # incremental
    python -m pageserve_b200.build --force    # rebuild everything

Each csrc/*.cu compiles to an object under pageserve_b200/_build/ (in
parallel, skipped when newer than its sources and headers), then nvcc links
the shared library next to this file. No GPU is needed to build.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libpageserve_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-I", str(ROOT / "include")] + ARCH


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objs = []
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or ptxas_info or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mtime):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda j: _compile(j[0], j[1], extra), jobs):
                if verbose or ptxas_info:
                    print(f"[nvcc] {obj.name}\n{log}", file=sys.stderr)
    newest = max(o.stat().st_mtime for o in objs)
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < newest:
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    build_torch_ops(force=force)
    return LIB


TORCH_OPS_SRC = PKG / "torch_ops" / "pageserve_ops.cpp"
TORCH_OPS_LIB = PKG / "libpageserve_torch_ops.so"


def build_torch_ops(force: bool = False) -> Path:
    """torch.ops.pageserve_b200.* (TORCH_LIBRARY registrations over the C
    ABI): one g++ compile against torch's headers, linked to
    libpageserve_b200.so (found next to it at run time) and torch's
    libraries."""
    import torch
    import torch.utils.cpp_extension as ce

    deps = [TORCH_OPS_SRC, ROOT / "include" / "pageserve_b200.h"]
    if (not force and TORCH_OPS_LIB.exists() and
            TORCH_OPS_LIB.stat().st_mtime >= max(d.stat().st_mtime for d in deps)):
        return TORCH_OPS_LIB
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = TORCH_OPS_LIB.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *incs,
           str(TORCH_OPS_SRC), "-o", str(tmp), f"-L{PKG}", "-lpageserve_b200", "-Wl,-rpath,$ORIGIN",
           *[f"-L{d}" for d in libdirs], *[f"-Wl,-rpath,{d}" for d in libdirs],
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch ops build failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TORCH_OPS_LIB)
    return TORCH_OPS_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers / spills / smem per kernel")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_info=a.ptxas_info))
