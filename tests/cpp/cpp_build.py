"""Build recipe of the C++ drop-in test programs (test infrastructure):
titan_block_test (the GPU test of include/ltm/titan_block.hpp) and the
pybind shim module of INTEGRATION.md (compiled on CPU to keep the snippet
honest).  Outputs go to tests/cpp/_build/.

    python tests/cpp/cpp_build.py [titan_block_test|pybind_shim]
"""
from __future__ import annotations

import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build"
LIBDIR = ROOT / "obsidian-memory-transformer_b200" / "ltm_b200"
CUDA = Path("/usr/local/cuda")


def _cxx() -> str:
    return shutil.which("g++") or "g++"


def _common() -> list[str]:
    return ["-std=c++17", "-O2", "-Wall", "-I" + str(ROOT / "include"), "-I" + str(CUDA / "include"),
            "-L" + str(LIBDIR), "-lltm_b200", "-Wl,-rpath," + str(LIBDIR),
            "-L" + str(CUDA / "lib64"), "-lcudart", "-Wl,-rpath," + str(CUDA / "lib64")]


def build_test() -> Path:
    OUT.mkdir(exist_ok=True)
    exe = OUT / "titan_block_test"
    src = HERE / "titan_block_test.cpp"
    hdr = ROOT / "include" / "ltm" / "titan_block.hpp"
    if exe.exists() and exe.stat().st_mtime >= max(src.stat().st_mtime, hdr.stat().st_mtime):
        return exe
    cmd = [_cxx(), str(src), "-o", str(exe)] + _common()
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"titan_block_test failed to build:\n{r.stdout}\n{r.stderr}")
    return exe


def build_pybind_shim() -> Path:
    import pybind11
    OUT.mkdir(exist_ok=True)
    ext = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    mod = OUT / ("ltm_pybind_shim" + ext)
    src = HERE / "pybind_shim.cpp"
    cmd = [_cxx(), "-shared", "-fPIC", str(src), "-o", str(mod),
           "-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"]] + _common()
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"pybind shim failed to build:\n{r.stdout}\n{r.stderr}")
    return mod


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "titan_block_test"
    print(build_pybind_shim() if what == "pybind_shim" else build_test())
