"""Build the in-tree CUDA library ``cactus_b200/libcactus_b200.so`` for sm_100a.

One nvcc invocation compiles every ``csrc/**/*.cu`` and ``csrc/**/*.cpp``:
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo --fmad=false``. ``--fmad=false``
keeps a*b+c unfused unless a kernel asks for fmaf() explicitly, which is how the
kernels reproduce the reference's rounding points.

Sources are relocatable device code (``-rdc=true``, linked with one device-link step) except
WHOLE_PROGRAM: tcgen05.mma kernels built as relocatable code read their shared-memory
operands from the wrong place (measured on B200 with nvcc 12.9: the same kernel and
descriptors give exact products as whole-program code and scrambled ones under -rdc), so
those files are compiled whole-program and reach the rest of the library through host
calls and kernel arguments only.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libcactus_b200.so")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"
WHOLE_PROGRAM = ("gemm_tc.cu",)


def sources():
    srcs = sorted(glob.glob(os.path.join(HERE, "csrc", "**", "*.cu"), recursive=True))
    srcs += sorted(glob.glob(os.path.join(HERE, "csrc", "**", "*.cpp"), recursive=True))
    return srcs


def _deps():
    files = sources()
    files += glob.glob(os.path.join(HERE, "csrc", "**", "*.cuh"), recursive=True)
    files += glob.glob(os.path.join(HERE, "csrc", "**", "*.h"), recursive=True)
    files += glob.glob(os.path.join(ROOT, "include", "**", "*.h"), recursive=True)
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _deps())


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> str:
    if not force and up_to_date():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    common = [ARCH, "-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "-I", os.path.join(ROOT, "include"),
              "-I", os.path.join(HERE, "csrc"), "--expt-relaxed-constexpr", "-diag-suppress=177"]
    if verbose:
        common += ["-Xptxas", "-v"]
    stamp = os.path.join(objdir, "flags.txt")
    flags_str = " ".join(common) + " rdc wp=" + ",".join(WHOLE_PROGRAM)
    if not os.path.exists(stamp) or open(stamp).read() != flags_str:
        force = True
    objs, procs = [], []
    jobs = jobs or max(1, min(8, os.cpu_count() or 1))
    for src in sources():
        rel = os.path.relpath(src, os.path.join(HERE, "csrc")).replace(os.sep, "_")
        obj = os.path.join(objdir, rel + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(f) for f in _deps()):
            continue
        rdc = [] if os.path.basename(src) in WHOLE_PROGRAM else ["-rdc=true"]
        cmd = [nvcc(), *common, *rdc, "-c", src, "-o", obj]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        while len([p for _, p in procs if p.poll() is None]) >= jobs:
            procs[0][1].wait() if procs[0][1].poll() is None else None
            import time
            time.sleep(0.2)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if out and (verbose or p.returncode):
            sys.stderr.write(out)
        if p.returncode:
            failed.append(src)
    if failed:
        raise RuntimeError(f"nvcc failed for: {failed}")
    with open(stamp, "w") as f:
        f.write(flags_str)
    tmp = LIB + ".tmp"
    subprocess.run([nvcc(), ARCH, "-rdc=true", "-shared", "-o", tmp, *objs, "-lpthread"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
