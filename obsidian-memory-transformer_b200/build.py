"""Build recipe of libltm_b200.so: every csrc/*.cu compiled for sm_100a with
nvcc and linked into ltm_b200/libltm_b200.so (in-tree, so it travels with the
repository snapshot).  Incremental: an object is rebuilt when its source or
any header under csrc/ or include/ is newer.

    python obsidian-memory-transformer_b200/build.py [--force] [-j N]
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
LIB = PKG / "ltm_b200" / "libltm_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-I" + str(ROOT / "include"),
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, obj: Path, verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stdout + r.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr_t = _headers_mtime()
    todo = []
    objs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_t):
            todo.append((s, o))
    jobs = jobs or min(len(todo) or 1, os.cpu_count() or 4)
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for obj, log in ex.map(lambda so: _compile(so[0], so[1], verbose), todo):
                logs.append((obj.name, log))
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc()] + ARCH + ["-shared", "-o", str(tmp)] + [str(o) for o in objs] + [
            "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        for name, log in logs:
            print(f"== {name}\n{log}")
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=a.v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
