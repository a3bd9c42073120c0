"""Build libkllm_cuda.so in-tree (sm_100a) with nvcc.

    python -m kmap_b200.build          # incremental
    python -m kmap_b200.build --force  # rebuild everything

Objects go to kmap_b200/_build/, the library to kmap_b200/libkllm_cuda.so.
The CUDA runtime is linked statically, so the library only needs the NVIDIA
driver at run time; the column-sharded decode talks to the other GPUs through
CUDA IPC mappings inside its own kernel, not through a collectives library.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(HERE, "libkllm_cuda.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall",
         "-I" + INCLUDE, "-I" + CSRC, "--expt-relaxed-constexpr"]


def sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    objs, changed = [], False
    for src in sources():
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.rsplit(".", 1)[0] + ".o")
        objs.append(o)
        if (not force and os.path.exists(o) and os.path.getmtime(o) >= os.path.getmtime(s)
                and os.path.getmtime(o) >= hdr):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", s, "-o", o]
        if src.endswith(".cu"):
            cmd += ["-Xptxas", "-v"] if verbose else []
        _run(cmd)
        changed = True
    if changed or force or not os.path.exists(LIB):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-Xlinker", "-Bsymbolic",
              "-Xlinker", "-soname=libkllm_cuda.so",
              "-lpthread", "-ldl", "-lrt"])
    return LIB


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError("nvcc failed for " + cmd[-1])
    if r.stderr.strip() and os.environ.get("KLLM_BUILD_VERBOSE"):
        sys.stderr.write(r.stderr)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
