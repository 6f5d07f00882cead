"""Build libtlmg.so, the sm_100a tier, in-tree with nvcc.

`python -m tierlm_b200.build` (or tierlm_b200.build.build()) compiles every
.cu file under csrc/ for sm_100a only and links one shared library next to
this file. The CUDA math discipline matches the reference's C flags
(-ffp-contract=off, no fast math): -fmad=false, IEEE division and square
root.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "libtlmg.so"
INCLUDE = HERE.parent / "include"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC,-O2,-fvisibility=default",
    "--expt-relaxed-constexpr",
]


# The persistent kernel runs 20 warps per SM (96 registers a thread); its
# per-step device functions are compiled separately under the same cap.
FILE_FLAGS = {"tlmg_fused.cu": ["-maxrregcount=96"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the sm_100a tier cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in deps())


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    cc = nvcc()
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [cc, *NVCC_FLAGS, *FILE_FLAGS.get(src.name, []), "-I", str(INCLUDE), "-dc", str(src), "-o", str(obj)]
        if ptxas_v:
            cmd[1:1] = ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs, "-o", str(tmp),
           "-lcudart", "-Xcompiler", "-fPIC"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="-v" in sys.argv)
    print(LIB)
