"""Build libiq.so (every .cu under csrc/) in-tree for sm_100a.

Run as ``python -m inferq_b200.build``.  Objects go to ``inferq_b200/_build``;
the shared library lands at ``inferq_b200/libiq.so`` so it travels with the
source tree.  Incremental: a source is recompiled when it or any header in
csrc/ or include/ is newer than its object.
"""
from __future__ import annotations

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
LIB = PKG / "libiq.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr",
              "-I" + str(ROOT / "include"), "-I" + str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, extra: list[str]) -> str:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = list(extra or [])
    hdr = _headers_mtime()
    srcs = sorted(CSRC.glob("*.cu"))
    todo = []
    objs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr):
            todo.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for (s, _), log in zip(todo, ex.map(lambda so: _compile(so[0], so[1], extra), todo)):
            if verbose and log.strip():
                print(f"[{s.name}]\n{log}", file=sys.stderr)
    if todo or not LIB.exists():
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart", "-lcuda", "-lnccl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    v = "-v" in sys.argv
    ex = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else []
    print(build(verbose=v or bool(ex), extra=ex))
