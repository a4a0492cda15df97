"""Build the b200q C-ABI library in-tree: ``_lib/libb200q.so`` (sm_100a).

Usage: ``python csrc/build.py [--verbose]``.  Rebuilds only when a source is
newer than the library.  nvcc cross-compiles, so no GPU is needed.  The
translation unit is compiled without --use_fast_math: the INT8 epilogue and the
quantizers rely on IEEE round-to-nearest fp32 arithmetic.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PACK = os.path.dirname(HERE)
ROOT = os.path.dirname(PACK)
OUT = os.path.join(PACK, "_lib", "libb200q.so")
SOURCES = ["capi.cu", "gemm8.cuh", "prologue.cuh", "qkv_rope.cuh", "quant.cuh", "w8a16.cuh", "w8a16_planes.cuh", "numerics.cuh", "ptx.cuh"]
HEADER = os.path.join(ROOT, "include", "b200q.h")


def nvcc_cmd(out=OUT, extra=()):
    nvcc = os.environ.get("NVCC", "nvcc")
    return [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
            "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
            "-o", out, os.path.join(HERE, "capi.cu"), *extra]


def up_to_date():
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = [os.path.join(HERE, s) for s in SOURCES] + [HEADER]
    return all(os.path.getmtime(d) <= t for d in deps if os.path.exists(d))


def build(force=False, verbose=False):
    if not force and up_to_date():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = nvcc_cmd()
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    msg = "\n".join(l for l in (r.stdout + r.stderr).splitlines()
                    if "compute_" not in l or "Warning" not in l)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{msg}")
    if verbose and msg.strip():
        print(msg)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
