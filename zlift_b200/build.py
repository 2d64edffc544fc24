"""Builds the native libraries of zlift_b200 in-tree with nvcc (sm_100a).

Outputs (under zlift_b200/lib/):
  libcublas.so.13   the cuBLAS-style C ABI and every CUDA kernel; soname
                    libcublas.so.13, plus the symlink libcublas.so -- the
                    file names zLift's loader interposition looks for
                    (zlift/src/install.rs:21-48, zblas/build.sh:47).
  libcudnn.so.9     re-exports the attention entry points from
                    libcublas.so.13 under the cuDNN library name (plus the
                    symlink libcudnn.so), since zLift loads a library by
                    that name for its DNN calls (zdnn/build.sh:15-17).

Usage: python -m zlift_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "lib")
BUILD = os.path.join(HERE, "_build")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-std=c++17", "-lineinfo", "--use_fast_math",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", os.path.join(ROOT, "include"),
]
# kernels whose arithmetic must not be relaxed by --use_fast_math
PRECISE = {"gemm_simt.cu", "gemm_tc.cu", "cublas_api.cu", "attn_f32.cu"}

SOURCES = [
    "gemm_tc.cu",
    "gemm_simt.cu",
    "fmha.cu",
    "attn_f32.cu",
    "attention_api.cu",
    "cublas_api.cu",
    "partition.cu",
    "noalloc.cu",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".h", ".cuh"))]
    deps.append(os.path.join(ROOT, "include"))
    if not force and os.path.exists(obj):
        t = os.path.getmtime(obj)
        newest = max(os.path.getmtime(d) for d in deps if os.path.exists(d))
        hdrs = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
        newest = max([newest] + [os.path.getmtime(h) for h in hdrs])
        if t >= newest:
            return obj
    flags = list(NVCC_FLAGS)
    if src in PRECISE:
        flags.remove("--use_fast_math")
    cmd = [nvcc()] + flags + ["-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def _link(objs: list[str]) -> None:
    out = os.path.join(LIB, "libcublas.so.13")
    tmp = out + ".tmp"
    cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + [
        "-Xlinker", "-soname=libcublas.so.13",
        "-Xlinker", "-Bsymbolic",
        "-Xlinker", "--no-undefined",
        "-ldl", "-lpthread",
    ]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    _symlink("libcublas.so.13", os.path.join(LIB, "libcublas.so"))

    # libcudnn.so.9: thin forwarding library
    src = os.path.join(CSRC, "cudnn_attention.c")
    dnn = os.path.join(LIB, "libcudnn.so.9")
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"), "-o",
           dnn + ".tmp", src, "-L", LIB, "-l:libcublas.so.13",
           "-Wl,-soname,libcudnn.so.9", "-Wl,-rpath,$ORIGIN", "-Wl,--no-undefined"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"libcudnn link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(dnn + ".tmp", dnn)
    _symlink("libcudnn.so.9", os.path.join(LIB, "libcudnn.so"))


def _symlink(target: str, link: str) -> None:
    if os.path.islink(link) or os.path.exists(link):
        os.remove(link)
    os.symlink(target, link)


def build(force: bool = False, jobs: int = 0) -> str:
    """Compiles and links the libraries; returns the path of libcublas.so.13."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    jobs = jobs or min(len(SOURCES), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), SOURCES))
    _link(objs)
    return os.path.join(LIB, "libcublas.so.13")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    a = ap.parse_args(argv)
    print(build(a.force, a.j))
    return 0


if __name__ == "__main__":
    sys.exit(main())
