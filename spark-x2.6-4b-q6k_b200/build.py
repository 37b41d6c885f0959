"""Build libspk.so (sm_100a) in-tree with nvcc.

The library is plain C-ABI: no torch types, no Python. It links the CUDA runtime
statically, so the .so travels to a GPU box with nothing else.

    python spark-x2.6-4b-q6k_b200/build.py [--verbose]   # -Xptxas -v register / spill report
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "spk", "libspk.so")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["common.cu", "vq.cu", "vq_mma.cu", "ggml.cu", "prefill.cu", "tp.cu", "attn.cu", "head_batch.cu", "q8t.cu", "vq_lut.cu", "vq_tab.cu", "vq_tc.cu", "draft.cu", "model.cu", "vqprof.cu"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-I", CSRC, "-I", os.path.join(ROOT, "include")]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed: " + " ".join(cmd))
    return r.stdout + r.stderr


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    objs = []
    log = ""
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdr_mtime = max([os.path.getmtime(h) for h in hdrs] + [0])
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if not force and not verbose and os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_mtime):
            continue
        extra = ["-Xptxas", "-v"] if verbose else []
        log += _run([NVCC, *ARCH, *FLAGS, *extra, "-dc" if False else "-c", s, "-o", o])
    newest = max(os.path.getmtime(o) for o in objs)
    if force or verbose or not os.path.exists(OUT) or os.path.getmtime(OUT) < newest:
        log += _run([NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-Xcompiler", "-fPIC", "-cudart", "static"])
    if verbose:
        print(log)
    return OUT


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv, force="--force" in sys.argv)
    print("built", OUT)
