"""Build recipe (test infrastructure only) of oracle/_ref/libref_kernels*.so:
the reference's own self-contained CUDA kernels, compiled from their source
lines where they lie in the reference tree, so the oracle can be checked
against the reference's arithmetic.

The reference as a whole does not compile (its Tensor header breaks every
translation unit), but these kernels depend only on cuda_runtime / cuda_fp16
and on type2float / cuda_cast from include/core/utils/cuda_utils.cuh, which
compiles once <memory> is included before it.  This recipe copies the cited
line ranges verbatim into oracle/_ref/ref_kernels_extracted.cuh (never into
the repository: oracle/_ref/ is git-ignored), checks that each range still
starts at the kernel it names, and compiles oracle/ref_launch.cu (the
launchers, written for this repository) against it twice:

* libref_kernels.so       with the reference's own CUDA flags (-O3
                          --use_fast_math, CMakeLists.txt:41-46): the kernels
                          as the reference ships them (approximate division,
                          rsqrtf, flush-to-zero);
* libref_kernels_ieee.so  with -O3 only: the same kernel bodies with IEEE
                          division and square root, the arithmetic the oracle
                          specifies for the quantizers.

Kernels (paths inside the reference project):
    linearQuantizeKernel        src/core/quantization/quantizer.cu:61-74
    symmetricQuantizeKernel     src/core/quantization/quantizer.cu:93-105
    perChannelQuantizeKernel    src/core/quantization/quantizer.cu:123-141
    perChannelDequantizeKernel  src/core/quantization/quantizer.cu:144-161
    layerNormResidualKernel     src/core/ops/fused_ops.cu:14-86
    biasActivationKernel        src/core/ops/fused_ops.cu:116-133
    GELU                        src/core/ops/fused_ops.cu:136-142
    storeStateKernel            src/core/ltm/memory_bank.cu:38-68

The reference tree is read from LTM_REFERENCE_ROOT, default /root/reference;
where it is absent (the GPU host) build() returns the prebuilt libraries, if
any, and never rebuilds them.

    python oracle/ref_kernels.py [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LAUNCH = HERE / "ref_launch.cu"
EXTRACTED = OUT / "ref_kernels_extracted.cuh"
LIBS = {"reference": OUT / "libref_kernels.so", "ieee": OUT / "libref_kernels_ieee.so"}
FLAGS = {"reference": ["-O3", "--use_fast_math"], "ieee": ["-O3"]}

# (file, first line, last line, the name the range must contain on its first
# two lines)
RANGES = [
    ("src/core/quantization/quantizer.cu", 61, 74, "linearQuantizeKernel"),
    ("src/core/quantization/quantizer.cu", 93, 105, "symmetricQuantizeKernel"),
    ("src/core/quantization/quantizer.cu", 123, 141, "perChannelQuantizeKernel"),
    ("src/core/quantization/quantizer.cu", 144, 161, "perChannelDequantizeKernel"),
    ("src/core/ops/fused_ops.cu", 14, 86, "layerNormResidualKernel"),
    ("src/core/ops/fused_ops.cu", 116, 133, "biasActivationKernel"),
    ("src/core/ops/fused_ops.cu", 136, 142, "struct GELU"),
    ("src/core/ltm/memory_bank.cu", 38, 68, "storeStateKernel"),
]


def reference_root() -> Path:
    return Path(os.environ.get("LTM_REFERENCE_ROOT", "/root/reference"))


def _nvcc() -> str:
    return os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"


def extract(ref: Path) -> str:
    parts = ["// Extracted verbatim from the reference tree by oracle/ref_kernels.py.\n"]
    for rel, a, b, name in RANGES:
        lines = (ref / rel).read_text().splitlines(keepends=True)
        chunk = lines[a - 1:b]
        head = "".join(chunk[:2])
        if name not in head or not chunk[-1].strip().startswith("}"):
            raise RuntimeError(f"{rel}:{a}-{b} no longer holds {name}; update the line range")
        parts.append(f"// ---- {rel}:{a}-{b}\n")
        parts.extend(chunk)
        parts.append("\n")
    return "".join(parts)


def build(force: bool = False) -> dict:
    """Returns {variant: path} of the libraries that exist after the build."""
    ref = reference_root()
    if not (ref / "src").is_dir():
        return {k: p for k, p in LIBS.items() if p.exists()}
    OUT.mkdir(exist_ok=True)
    text = extract(ref)
    if not EXTRACTED.exists() or EXTRACTED.read_text() != text:
        EXTRACTED.write_text(text)
    src_t = max(EXTRACTED.stat().st_mtime, LAUNCH.stat().st_mtime, Path(__file__).stat().st_mtime)
    for variant, lib in LIBS.items():
        if not force and lib.exists() and lib.stat().st_mtime >= src_t:
            continue
        tmp = lib.with_suffix(".so.tmp")
        cmd = [_nvcc(), "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
               *FLAGS[variant], "-Xcompiler", "-fPIC", "-shared",
               "-I" + str(OUT), "-I" + str(ref / "include"), str(LAUNCH), "-o", str(tmp)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"reference kernels ({variant}) failed to build:\n{r.stdout}\n"
                               f"{r.stderr}")
        tmp.replace(lib)
    return dict(LIBS)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
