"""Builds libiconnx_b200.so in-tree with nvcc for sm_100a.

    python -m iconnx_b200.build          # or iconnx_b200.build.build()

Every .cu / .cpp under csrc/ is compiled with relocatable device code and
linked into one shared library next to this file.  No NVRTC, no JIT cache:
the built .so travels with the source tree.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libiconnx_b200.so")
BUILD_DIR = os.path.join(HERE, "_build")

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"] + ARCH


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _deps() -> list[str]:
    return (_sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(HERE, "..", "include", "*.h")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, jobs: int = 8) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    procs = []
    for src in _sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        objs.append(obj)
        cmd = [NVCC, *NVCC_FLAGS, "-c", src, "-o", obj]
        if os.environ.get("ICX_PTXAS_VERBOSE"):
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        if len(procs) >= jobs:
            _drain(procs)
    _drain(procs)
    link = [NVCC, *ARCH, "-shared", "-rdc=true", "-o", OUT, *objs, "-lcudart", "-lcublas"]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout)
    return OUT


def _drain(procs):
    errs = []
    for src, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            errs.append(f"{src}:\n{text}")
        elif text.strip() and os.environ.get("ICX_PTXAS_VERBOSE"):
            print(text, file=sys.stderr)
    procs.clear()
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(OUT)
