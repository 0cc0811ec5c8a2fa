"""Build the in-tree CUDA library (and, for tests, the oracle).

    python -m memvanta_b200.build            # libmemvanta_b200.so (sm_100a)
    python -m memvanta_b200.build --oracle   # also oracle/ (+ oracle/_ref when the reference checkout exists)
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def build_lib(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(HERE, "csrc")], check=True)
    return os.path.join(HERE, "libmemvanta_b200.so")


# Checkout of the reference sources the oracle's reference build compiles
# (test infrastructure only); MV_REFERENCE_DIR overrides the default.
REF_ROOT = os.environ.get("MV_REFERENCE_DIR", "/root/reference")


def build_oracle(ref_root: str | None = None, jobs: int = 8) -> None:
    ref_root = ref_root or REF_ROOT
    args = ["make", "-s", f"-j{jobs}", "-C", os.path.join(ROOT, "oracle")]
    if os.path.isdir(ref_root):
        args.append(f"REF={ref_root}")
    else:
        args.append("oracle")  # the reference is absent: only the C restatement
    subprocess.run(args, check=True)


if __name__ == "__main__":
    build_lib()
    if "--oracle" in sys.argv:
        build_oracle()
