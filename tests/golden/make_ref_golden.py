"""Generates tests/golden/reference_kernels.npz (test infrastructure): runs
every case of ref_cases.py through the reference's own kernels, compiled by
oracle/ref_kernels.py from the reference's sources, in both builds (the
reference's flags and the IEEE build), on cuda:0, and stores their outputs.

    python tests/golden/make_ref_golden.py [--out PATH]

Needs a GPU and oracle/_ref/libref_kernels*.so.  The CPU suite checks the
oracle against the stored outputs; the GPU suite re-runs the kernels and
checks that they reproduce them bit for bit.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
for p in (str(ROOT), str(HERE)):
    if p not in sys.path:
        sys.path.insert(0, p)

import ref_cases  # noqa: E402


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(ref_cases.FIXTURE))
    a = ap.parse_args()
    from oracle import oracle
    libs = {v: ref_cases.load(v) for v in ref_cases.VARIANTS}
    arrays = {}
    for name, (kind, dt, shape, seed) in ref_cases.CASES.items():
        inp = ref_cases.inputs(name)
        for variant, lib in libs.items():
            out = ref_cases.run(lib, name, inp, oracle)
            arrays[f"{name}/{variant}"] = out.astype(np.float16) if (
                dt == "f16" and out.dtype != np.int8) else out
    np.savez_compressed(a.out, **arrays)
    print(f"wrote {len(arrays)} arrays to {a.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
