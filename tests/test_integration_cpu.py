"""The integration artefacts a pickle maintainer applies (no GPU):

* lestramanika_b200/hook/pickle_makefile_cuda.patch adds the PICKLE_CUDA=1
  target to the reference's Makefile (Makefile:27-54 of the reference): an
  nvcc rule over every .cu of lestramanika_b200/csrc (the same translation
  units lestramanika_b200/build.py compiles), the hook glue, the library
  link;
* lestramanika_b200/hook/pickle_fast_cuda_hook.patch applies to
  src/pickle_fast.c.
Both are applied to temporary copies; the reference's own build is not run."""
import glob
import os
import shutil
import subprocess

import pytest

import __graft_entry__
from lestramanika_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOOK = os.path.join(ROOT, "lestramanika_b200", "hook")
REF = os.environ.get("PICKLE_REF") or __graft_entry__.REFERENCE_MOUNT


def _patched(src, patch, tmp_path):
    if not os.path.exists(src):
        pytest.skip("the reference's sources are not mounted here")
    out = tmp_path / os.path.basename(src)
    r = subprocess.run(["patch", "-s", "-o", str(out), src], stdin=open(patch), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out.read_text()


def test_makefile_patch_adds_the_nvcc_target(tmp_path):
    mk = _patched(os.path.join(REF, "Makefile"), os.path.join(HOOK, "pickle_makefile_cuda.patch"), tmp_path)
    block = mk[mk.index("ifeq ($(PICKLE_CUDA),1)"):]
    block = block[:block.index("endif")]
    assert "$(wildcard $(PICKLE_CUDA_PKG)/csrc/*.cu)" in block
    assert "arch=compute_100a,code=sm_100a" in block
    assert "-DPICKLE_CUDA" in block and "src/pickle_cuda_hook.o" in block and "-lpickle_cuda" in block
    assert ".DEFAULT_GOAL    := all" in block
    # the wildcard covers exactly the translation units the in-tree build compiles
    cu = sorted(os.path.basename(p) for p in glob.glob(os.path.join(ROOT, "lestramanika_b200", "csrc", "*.cu")))
    assert cu == sorted(build.UNITS)


def test_pickle_fast_patch_applies_and_hooks_the_attention_block(tmp_path):
    src = _patched(os.path.join(REF, "src", "pickle_fast.c"), os.path.join(HOOK, "pickle_fast_cuda_hook.patch"),
                   tmp_path)
    assert src.count("#ifdef PICKLE_CUDA") == 3
    assert "pickle_cuda_hook_auto(state, L, pos, q, k, v, ao)" in src
    assert "__attribute__((weak))" in src
    assert shutil.which("patch")
