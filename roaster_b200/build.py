"""Build libroaster_b200.so in-tree: every CUDA source under csrc/ for sm_100a with nvcc.

Usage: python -m roaster_b200.build   (or roaster_b200.build.build())
The shared library links the CUDA runtime statically, so loading it needs no GPU; calling a
compute entry point without a B200 returns -1.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libroaster_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-fopenmp", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    cand = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cand, "bin", "nvcc")
    return path if os.path.exists(path) else (shutil.which("nvcc") or "nvcc")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    deps.append(os.path.join(HERE, "..", "include", "roaster_cuda.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        if not os.path.exists(SLOT_LIB) or os.path.getmtime(SLOT_LIB) < max(os.path.getmtime(SLOT_SRC),
                                                                            os.path.getmtime(LIB)):
            build_slot_threads()
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                            text=True)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append(f"{src}:\n{out}")
        elif verbose and out:
            print(out)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-Xcompiler", "-fPIC", "-lgomp"]
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("link failed:\n" + out.stdout + out.stderr)
    os.replace(tmp, LIB)
    build_slot_threads()
    return LIB


SLOT_SRC = os.path.join(HERE, "slot_threads.c")
SLOT_LIB = os.path.join(HERE, "libslot_threads.so")


def build_slot_threads() -> str:
    """libslot_threads.so: native slot threads for driving the step group (slot_threads.c),
    linked against libroaster_b200.so in the same folder."""
    inc = os.path.join(HERE, "..", "include")
    tmp = SLOT_LIB + ".tmp"
    cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-Werror", "-fPIC", "-shared", "-I", inc, SLOT_SRC,
           "-o", tmp, "-L", HERE, "-l:libroaster_b200.so", "-Wl,-rpath,$ORIGIN", "-lpthread"]
    out = subprocess.run(cmd, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("slot_threads build failed:\n" + out.stdout + out.stderr)
    os.replace(tmp, SLOT_LIB)
    return SLOT_LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
