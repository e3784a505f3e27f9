"""Builds libengram_b200.so (the C-ABI library of the CUDA path) in-tree with nvcc,
for sm_100a only.  `python -m engraft_ngram_b200.build [-v]`."""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libengram_b200.so"
SOURCES = ["engram_table.cu", "engram_forward.cu", "engram_backward.cu", "engram_adam.cu", "engram_shard.cu", "engram_scan.cu",
           "engram_rowset.cu", "engram_stage.cu", "engram_ple.cu", "engram_gemm.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found: the CUDA path needs the CUDA toolkit to build")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, out: Path | None = None, defines=()) -> Path:
    """Compiles the library (to `out`, default the in-tree libengram_b200.so);
    `defines` are extra -D tuning macros."""
    target = Path(out) if out is not None else LIB
    if out is None and not force and not needs_build():
        return LIB
    cmd = [nvcc(), *ARCH, *(f"-D{d}" for d in defines), "-lineinfo", "-O3", "-std=c++17", "--shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE), "-I", str(CSRC),
           *(str(CSRC / s) for s in SOURCES), "-o", str(target) + ".tmp", "-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(target) + ".tmp", target)
    return target


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force=True)
    print(LIB)
