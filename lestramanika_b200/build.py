"""Build the B200 attention library in-tree.

    python -m lestramanika_b200.build          # libpickle_cuda.so
    python -m lestramanika_b200.build --all    # + oracle/ checkers

The library is compiled with nvcc for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`) into
lestramanika_b200/libpickle_cuda.so, next to this file, so it travels with
the source tree. No fast-math: expf/sinf keep full precision.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libpickle_cuda.so")
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_lib(force=False, verbose=False):
    deps = _sources() + [os.path.join(ROOT, "include", "pickle_cuda.h"), __file__]
    if not force and not _stale(LIB, deps):
        return LIB
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
           "-DPICKLE_CUDA_BUILD", "-o", LIB + ".tmp", os.path.join(CSRC, "pickle_cuda.cu"),
           os.path.join(CSRC, "decode_noalloc.cu"), os.path.join(CSRC, "peer_xchg.cu"), os.path.join(CSRC, "matvec.cu"),
           os.path.join(CSRC, "forward.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_oracle(with_cuda_harness=True):
    """Build the parity checkers under oracle/ (test infrastructure)."""
    ref = os.environ.get("PICKLE_REF", "/root/reference")
    make = ["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={ref}"]
    subprocess.run(make + ["oracle"], check=True)
    if os.path.isdir(os.path.join(ref, "src")):
        subprocess.run(make + ["ref"], check=True)
        if with_cuda_harness:
            subprocess.run(make + ["cuda"], check=True)


if __name__ == "__main__":
    build_lib(force="--force" in sys.argv, verbose="-v" in sys.argv)
    if "--all" in sys.argv:
        build_oracle()
    print(LIB)
