"""Builds libtfx.so in-tree with nvcc for sm_100a (no GPU needed).

    python tenferro-decision-rs_b200/build.py [--force] [--verbose-ptxas]

Objects go to tenferro-decision-rs_b200/_build/, the library to
tenferro-decision-rs_b200/lib/libtfx.so. --fmad=false keeps every a*b+c in the
kernels as two roundings unless the source asks for a fused multiply-add, as
the reference's Rust (which never contracts) computes it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libtfx.so")
INCLUDE = os.path.join(ROOT, "include")

SOURCES = ["runtime.cu", "elementwise.cu", "norms.cu", "softmax.cu", "rope.cu", "session.cu",
           "rms_stream.cu", "attention.cu", "embedding.cu", "gemm_epilogue.cu"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", "--extended-lambda",
    "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; libtfx needs the CUDA 12.9 toolchain")
    return path


def _headers() -> list[str]:
    hs = [os.path.join(INCLUDE, "tfx.h")]
    hs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose_ptxas: bool, force: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.splitext(os.path.basename(src))[0] + ".o")
    if not force and not _stale(obj, [src] + _headers()):
        return obj, ""
    cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + [
        "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        futs = [ex.submit(_compile, s, verbose_ptxas, force) for s in srcs]
        objs = []
        for f in futs:
            obj, log = f.result()
            objs.append(obj)
            if log:
                logs.append(log)
    if force or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    if verbose_ptxas:
        sys.stderr.write("".join(logs))
    return LIB


def main(argv: list[str]) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
