"""Build libeii.so (and the eii_check CLI) in-tree for sm_100a with nvcc.

    python exact-integer-inference_b200/build.py [--force]

Outputs next to this file: libeii.so (the C ABI of include/eii.h) and eii_check (the drop-in for
the reference's `intref VECTORDIR [MODELDIR]` checkers).  Rebuilds only when a source is newer.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB = os.path.join(HERE, "libeii.so")
CLI = os.path.join(HERE, "eii_check")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = os.environ.get("NVCC", "nvcc")


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".c", ".h"))] + \
        [os.path.join(INCLUDE, "eii.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False):
    deps = _sources()
    if force or _stale(LIB, deps):
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O2",
               "-I" + INCLUDE, "-I" + CSRC, "-o", LIB, os.path.join(CSRC, "eii_engine.cu")]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    cli_src = os.path.join(CSRC, "eii_check.c")
    if os.path.exists(cli_src) and (force or _stale(CLI, [cli_src, LIB])):
        cmd = ["gcc", "-O2", "-Wall", "-Wextra", "-I" + INCLUDE, "-o", CLI, cli_src, "-L" + HERE, "-leii",
               "-Wl,-rpath,$ORIGIN"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    build(a.force, verbose=True)
    sys.exit(0)
