"""B200-native GQA attention block for pickle (lee-muriithi-kingori/lestramanika).

The product is libpickle_cuda.so (C ABI: include/pickle_cuda.h) built from
lestramanika_b200/csrc for sm_100a; this package loads it (api), shards it
across GPUs (dist), runs a prompt's attention half of a layer
(prefill_layer) or the whole forward pass of a GGUF model (model, gguf) on
the device, and holds the pickle_fast.c integration hook (hook/).
"""
from .api import (PickleCuda, PickleError, lse_merge_dev, lse_merge_packed_dev, abi_version, lib,  # noqa: F401
                  PREFILL_F32, PREFILL_BF16)
