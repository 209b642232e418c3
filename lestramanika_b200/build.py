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


UNITS = ("pickle_cuda.cu", "decode_noalloc.cu", "peer_xchg.cu", "matvec.cu", "forward.cu")


def build_lib(force=False, verbose=False):
    """Compile each translation unit to an object (in parallel), then link
    the shared library; objects go to a build folder next to the library."""
    from concurrent.futures import ThreadPoolExecutor
    deps = _sources() + [os.path.join(ROOT, "include", "pickle_cuda.h"), __file__]
    if not force and not _stale(LIB, deps):
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
             "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-DPICKLE_CUDA_BUILD"]
    if verbose:
        flags.insert(0, "-Xptxas=-v")

    def compile_unit(unit):
        obj = os.path.join(objdir, unit.replace(".cu", ".o"))
        subprocess.run([NVCC, *flags, "-c", "-o", obj, os.path.join(CSRC, unit)], check=True)
        return obj

    with ThreadPoolExecutor(max_workers=len(UNITS)) as pool:
        objs = list(pool.map(compile_unit, UNITS))
    subprocess.run([NVCC, *ARCH, "-shared", "-o", LIB + ".tmp", *objs], check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


def build_oracle(with_cuda_harness=True, ref=None):
    """Build the parity checkers under oracle/ (test infrastructure). The
    reference's own objects are compiled only when its sources are given
    (`ref`, or the PICKLE_REF environment variable)."""
    ref = ref or os.environ.get("PICKLE_REF", "")
    make = ["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={ref}"]
    subprocess.run(make + ["oracle"], check=True)
    if ref and os.path.isdir(os.path.join(ref, "src")):
        subprocess.run(make + ["ref"], check=True)
        if with_cuda_harness:
            subprocess.run(make + ["cuda"], check=True)


if __name__ == "__main__":
    build_lib(force="--force" in sys.argv, verbose="-v" in sys.argv)
    if "--all" in sys.argv:
        build_oracle(ref=next((a.split("=", 1)[1] for a in sys.argv if a.startswith("--ref=")), None))
    print(LIB)
