"""TEST INFRASTRUCTURE: build recipe for the oracle.

* ``libstrata_oracle.so`` — the C restatement (oracle/strata_oracle.c), always built.
* ``_ref/libstrata_ref.so`` — the reference's own kernels/strata.cu compiled natively with
  g++ where it lies (never copied), behind oracle/ref_shim.hpp + oracle/ref_runtime.cpp.
  Built only when the reference tree is present (this container); the .so then travels
  with the repository snapshot. Outputs go to oracle/_ref/ only.

Both use -ffp-contract=off: the reference's WASM target has no fused multiply-add, so every
product and sum rounds separately there, and must here.
"""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "libstrata_oracle.so"
REF_DIR = HERE / "_ref"
REF_SO = REF_DIR / "libstrata_ref.so"
REFERENCE_ROOT = pathlib.Path(os.environ.get("STRATA_REFERENCE_ROOT", str(pathlib.Path(__file__).resolve().parents[2] / "reference")))
REF_SOURCE = REFERENCE_ROOT / "kernels" / "strata.cu"
FP_FLAGS = ["-ffp-contract=off", "-fno-fast-math"]


def _newer(target: pathlib.Path, *sources: pathlib.Path) -> bool:
    return target.exists() and all(target.stat().st_mtime >= s.stat().st_mtime for s in sources)


def build_oracle(force: bool = False) -> pathlib.Path:
    src = HERE / "strata_oracle.c"
    if force or not _newer(ORACLE_SO, src, HERE / "strata_expf.h"):
        cmd = ["gcc", "-O2", "-fPIC", "-shared", *FP_FLAGS, "-o", str(ORACLE_SO), str(src), "-lm"]
        subprocess.run(cmd, check=True)
    return ORACLE_SO


def build_ref(force: bool = False) -> pathlib.Path | None:
    """Compile the reference's kernels/strata.cu natively; None when the reference is absent."""
    if not REF_SOURCE.exists():
        return REF_SO if REF_SO.exists() else None
    srcs = [HERE / "ref_runtime.cpp", HERE / "ref_shim.hpp", REF_SOURCE]
    if force or not _newer(REF_SO, *srcs):
        REF_DIR.mkdir(exist_ok=True)
        cmd = ["g++", "-O3", "-std=c++20", "-fPIC", "-shared", "-pthread", *FP_FLAGS, "-w",
               "-include", str(HERE / "ref_shim.hpp"), f'-DSTRATA_REF_SOURCE="{REF_SOURCE}"',
               "-I", str(HERE), "-o", str(REF_SO), str(HERE / "ref_runtime.cpp")]
        subprocess.run(cmd, check=True)
    return REF_SO


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_oracle(force))
    print(build_ref(force))
