"""Build libnfx.so (the C-ABI library with every sm_100a kernel) in-tree.

    python -m neuroflow_b200.build [-v]

Compiles neuroflow_b200/csrc/*.cu and *.cpp with nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a), objects under _build/, and links
neuroflow_b200/libnfx.so and the nflow_infer command-line front-end next to it.  The CUDA runtime is linked statically so the library does
not depend on which libcudart the host process (e.g. torch) loaded.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(ROOT, "_build", "nfx")
LIB = os.path.join(PKG, "libnfx.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "nfx.h"))
    return max(os.path.getmtime(h) for h in hs if os.path.exists(h))


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if (os.path.exists(obj) and os.path.getmtime(obj) >= os.path.getmtime(src)
            and os.path.getmtime(obj) >= _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    if src.endswith(".cpp"):
        cmd += ["-x", "cu"] if False else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if (not os.path.exists(LIB)
            or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs)):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    _build_cli()
    return LIB


CLI_SRC = os.path.join(PKG, "cli", "nflow_infer.cpp")
CLI = os.path.join(PKG, "nflow_infer")


def _build_cli() -> None:
    """The nflow_infer executable, linked against libnfx.so (found next to it)."""
    hpp = os.path.join(ROOT, "include", "nflow_runtime.hpp")
    if os.path.exists(CLI) and os.path.getmtime(CLI) >= max(os.path.getmtime(CLI_SRC),
                                                              os.path.getmtime(LIB),
                                                              os.path.getmtime(hpp)):
        return
    cmd = ["g++", "-std=c++17", "-O2", "-I" + os.path.join(ROOT, "include"), CLI_SRC, "-o", CLI,
           "-L" + PKG, "-lnfx", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nflow_infer build failed:\n{r.stdout}\n{r.stderr}")


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
