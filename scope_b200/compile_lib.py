"""Compile libscope_b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m scope_b200.compile_lib [-v]

Objects are compiled in parallel into scope_b200/_build/ and linked with the
static CUDA runtime; the library links nothing from PyTorch.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libscope_b200.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
              "-Xptxas", "-v", "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    for cand in (os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    # nvcc picks the host compiler from PATH; the system gcc links OpenMP-free C++ fine.
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)
    out = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if out.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{out.stdout}\n{out.stderr}")
    return obj, out.stderr if verbose else ""


def build(verbose: bool = False, force: bool = False) -> str:
    """Build the library if any source is newer than it; return its path."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    newest = max([os.path.getmtime(s) for s in srcs] + [_headers_mtime()])
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [r[0] for r in results]
    if verbose:
        for _, log in results:
            sys.stdout.write(log)
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB + ".tmp", *objs, "-lcuda" if False else "-ldl"]
    env = dict(os.environ)
    env.pop("CC", None)
    env.pop("CXX", None)
    out = subprocess.run(cmd, capture_output=True, text=True, env=env)
    if out.returncode != 0:
        raise RuntimeError(f"link failed:\n{out.stdout}\n{out.stderr}")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
