"""Build the CUDA library ``libg4b.so`` in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in
parallel), then linked into ``g4b/libg4b.so`` next to this file, so the built
library travels with the source tree.  Nothing is JIT-compiled or cached
outside the repository.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                       # the gemma4-12b-snapdragonx2elite_b200 directory
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libg4b.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fvisibility=hidden", "-DG4B_BUILDING=1"]


def nvcc_path() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the g4b CUDA library cannot be built")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(d) <= t for d in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; return its path.

    Processes that load the library at the same time (one per GPU rank) build
    it at most once: the build holds an exclusive lock on a file in the build
    directory and re-checks freshness once it has the lock."""
    if not force and up_to_date():
        return LIB_PATH
    import fcntl
    os.makedirs(BUILD_DIR, exist_ok=True)
    with open(os.path.join(BUILD_DIR, ".lock"), "w") as lockf:
        fcntl.flock(lockf, fcntl.LOCK_EX)
        try:
            if not force and up_to_date():
                return LIB_PATH
            return _build_locked(verbose, ptxas_verbose)
        finally:
            fcntl.flock(lockf, fcntl.LOCK_UN)


def _build_locked(verbose: bool, ptxas_verbose: bool) -> str:
    nvcc = nvcc_path()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src: str) -> tuple[str, str]:
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return obj, r.stdout + r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, sources()))
    if verbose or ptxas_verbose:
        for _, log in results:
            if log.strip():
                print(log)
    objs = [o for o, _ in results]
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose=True, ptxas_verbose="--ptxas-v" in sys.argv))
