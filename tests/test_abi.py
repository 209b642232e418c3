"""The C ABI library loads and exports every entry point of include/*.h (no GPU calls)."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

import lestramanika_b200 as L
from lestramanika_b200 import api

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names.update(re.findall(r"^PICKLE_CUDA_API\s+[\w\s\*]+?\b(pickle_cuda_\w+)\s*\(", src, re.M))
    return names


def test_header_declares_entry_points():
    d = _declared()
    for must in ("pickle_cuda_init", "pickle_cuda_free", "pickle_cuda_attn_decode", "pickle_cuda_attn_prefill",
                 "pickle_cuda_decode_batch_dev", "pickle_cuda_prefill_dev", "pickle_cuda_decode_partial_dev",
                 "pickle_cuda_lse_merge_dev"):
        assert must in d


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(api.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", api.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s(pickle_cuda_\w+)", out))
    assert exported == _declared()


def test_python_mirror_covers_the_abi():
    assert set(api.SIGNATURES) == _declared()


def test_abi_version():
    assert L.abi_version() == 1


def test_error_names_mirror_pickle_codes():
    assert api.ERROR_NAMES[-7] == "PICKLE_ERR_RANGE" and api.ERROR_NAMES[-9] == "PICKLE_ERR_DEVICE"
    e = api.PickleError(-6, "x")
    assert e.code == -6 and "PICKLE_ERR_ARG" in str(e)


def test_hook_patch_is_minimal():
    """The integration patch only adds lines to pickle_fast.c, all under PICKLE_CUDA."""
    patch = open(os.path.join(ROOT, "lestramanika_b200", "hook", "pickle_fast_cuda_hook.patch")).read()
    body = [l for l in patch.splitlines() if l.startswith(("+", "-")) and not l.startswith(("+++", "---"))]
    assert all(l.startswith("+") for l in body)
    assert sum(l.startswith("+#ifdef PICKLE_CUDA") for l in body) == 3


def test_python_handles_have_their_methods():
    """The Python mirror's handle classes expose every call the tests and the bench use."""
    for name in ("handle", "open", "attach", "set_wait", "buffer", "put", "sync", "close"):
        assert callable(getattr(api.PeerExchange, name, None)), name
    for name in ("decode_batch_dev", "decode_gather_dev", "decode_seqshard_dev", "decode_partial_dev",
                 "prefill_dev", "sync", "close", "kv_tensors"):
        assert callable(getattr(api.PickleCuda, name, None)), name
    assert callable(api.decode_xchg_bytes)
