"""Build the C-ABI shared library libspecdec_b200.so in-tree (sm_100a only).

    python adaptive-specdec_b200/build.py [-v]

The library is written next to this file so it travels with the source tree
(no JIT cache, no site-packages install).  It links only the CUDA runtime.
"""
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
LIB = HERE / "libspecdec_b200.so"

SOURCES = ["sd_sampling.cu", "sd_kvcache.cu", "sd_attention.cu", "sd_shard.cu", "sd_layers.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and pathlib.Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def up_to_date():
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return all(d.stat().st_mtime <= t for d in deps)


def build(verbose=False, force=False):
    """Compile every .cu source into one shared library; returns its path."""
    if not force and up_to_date():
        return LIB
    objs = []
    build_dir = HERE / "_build"
    build_dir.mkdir(exist_ok=True)
    for src in sources():
        obj = build_dir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src),
               "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs, "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
