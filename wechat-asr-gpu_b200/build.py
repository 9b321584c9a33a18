"""Build libwasr_gpu.so in-tree for sm_100a (nvcc, no JIT cache).

Every .cu under csrc/ is compiled with `-gencode arch=compute_100a,code=sm_100a -lineinfo`
and linked into one shared library next to this file.  Host code is compiled with
-ffp-contract=off so the host fbank keeps the reference's floating-point order.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "libwasr_gpu.so")
SOURCES = ["gemm.cu", "kern.cu", "ctx.cu", "engine.cu", "fbank.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _ccbin() -> list[str]:
    # the system g++ carries libgomp; an alternative compiler on PATH may not
    return ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []


def _flags() -> list[str]:
    return ARCH + _ccbin() + [
        "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fopenmp,-ffp-contract=off",
        "-I", os.path.join(HERE, "..", "include"), "-I", CSRC,
    ]


def _stale(obj: str, src: str) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps += [os.path.join(HERE, "..", "include", f) for f in ("wtlgpu.h", "wasr.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    jobs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        if force or _stale(obj, src):
            jobs.append([nvcc, *_flags(), "-c", src, "-o", obj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, file=sys.stderr)
        return r

    with cf.ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        list(ex.map(run, jobs))
    objs = [os.path.join(BUILD, s.replace(".cu", ".o")) for s in SOURCES]
    if jobs or not os.path.exists(OUT) or any(os.path.getmtime(o) > os.path.getmtime(OUT) for o in objs):
        run([nvcc, *ARCH, *_ccbin(), "-shared", "-o", OUT, *objs, "-Xcompiler", "-fopenmp", "-lgomp"])
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
