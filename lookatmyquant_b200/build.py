"""Builds liblamq_b200.so, the C-ABI library of sm_100a kernels, in-tree with nvcc.

    python -m lookatmyquant_b200.build          # incremental
    python -m lookatmyquant_b200.build --force  # rebuild everything

Every `csrc/*.cu` file is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`), with -lineinfo for
profiling, and linked into `lookatmyquant_b200/liblamq_b200.so`; objects go to `lookatmyquant_b200/_build/`.
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
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "liblamq_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(exe).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build liblamq_b200.so")
    return exe


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "lamq_b200.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in _deps(src))


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(-4, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    todo = [(s, BUILD / (s.stem + ".o")) for s in srcs if force or _stale(BUILD / (s.stem + ".o"), s)]
    logs = {}
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, verbose): s for s, o in todo}
            for f in cf.as_completed(futs):
                logs[futs[f].name] = f.result()
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        for name, log in sorted(logs.items()):
            print(f"== {name}\n{log}", file=sys.stderr)
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true", help="print ptxas register/spill reports")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
