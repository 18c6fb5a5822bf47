"""Build the sm_100a shared library ``libadaattn_b200.so`` in-tree with nvcc.

Each ``csrc/*.cu`` compiles to an object file under ``_build/`` (in parallel),
then one link produces the library next to this file. The CUDA runtime is
linked statically; the driver API (tensor-map encoding) is resolved at run
time through ``cudaGetDriverEntryPointByVersion``, so no libcuda stub is
needed at link time and the library cross-compiles on a machine without a GPU.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(os.path.dirname(PKG), "_build")
LIB = os.path.join(PKG, "libadaattn_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills",
    "-DNDEBUG",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    out = []
    for d in (CSRC, os.path.join(os.path.dirname(PKG), "include")):
        out += [os.path.join(d, f) for f in os.listdir(d)]
    out.append(os.path.abspath(__file__))
    return out


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    """Compile (if needed) and return the path of the shared library."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    flags = NVCC_FLAGS + list(extra_flags or [])
    deps = _deps()
    objs = []
    jobs = []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, deps):
            jobs.append([nvcc] + flags + ["-c", src, "-o", obj])

    def run(cmd):
        res = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, res

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for cmd, res in ex.map(run, jobs):
                if verbose or res.returncode != 0:
                    sys.stderr.write(res.stdout + res.stderr)
                if res.returncode != 0:
                    raise RuntimeError(f"nvcc failed: {' '.join(cmd)}")
    if force or jobs or _stale(LIB, objs):
        cmd = [nvcc] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
