"""Build the C-ABI shared library ``libllmopt_b200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` (git-ignored)
and linked with a static CUDA runtime, so the library does not depend on which
``libcudart`` torch happens to load.  The build is incremental: objects are
rebuilt when their source or any header in ``csrc/`` or ``include/`` changed.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD = os.path.join(REPO_DIR, "_build")
LIB_NAME = "libllmopt_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", CSRC, "-I", INCLUDE,
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build llmopt_b200")


def _headers_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    files += glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(f) for f in files), default=0.0)


def _compile(nvcc: str, src: str, obj: str, verbose: bool) -> None:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile and link the library if anything changed; return its path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_time = _headers_mtime()
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = (force or not os.path.exists(obj)
                 or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_time))
        if stale:
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 1)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose) for s, o in jobs]
            for f in futs:
                f.result()
    newest = max(os.path.getmtime(o) for o in objs)
    if force or jobs or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < newest:
        tmp = LIB_PATH + ".tmp"
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", tmp, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
