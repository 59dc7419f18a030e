"""Builds ``libtopos_b200.so`` in-tree with nvcc for sm_100a.

Host files (``csrc/*.cpp``) and CUDA files (``csrc/*.cu``) compile to objects
under ``_build/`` in parallel, then link into one shared library with a static
CUDA runtime, the driver API and NVRTC.  NCCL is loaded at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(ROOT, "_build")
OUT = os.path.join(HERE, "libtopos_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off",
          f"-I{os.path.join(ROOT, 'include')}", "-I/usr/local/cuda/include"]


def _compile(src: str) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    deps = [src] + glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(ROOT, "include", "topos_b200.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", src, "-o", obj]
    if src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"] if os.environ.get("TB_PTXAS_VERBOSE") else []
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    if res.stderr.strip() and os.environ.get("TB_PTXAS_VERBOSE"):
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cpp")) + glob.glob(os.path.join(CSRC, "*.cu")))
    if force:
        for obj in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(obj)
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objects = list(pool.map(_compile, sources))
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= max(os.path.getmtime(o) for o in objects)):
        return OUT
    cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objects, "-L/usr/local/cuda/lib64",
           "-lnvrtc", "-ldl", "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
