"""mini_llama_b200: B200 (sm_100a) implementation of mini_llama's decode and
prefill hot path.

The product is the CUDA shared library built from csrc/ (C ABI in
include/mlb.h) plus the C++17 adapter in adapter/ that implements mini_llama's
own CUDA-op headers on top of it.  The Python modules here are bindings used by
the tests and the benchmark.
"""
from .capi import Lib, MlbError, load  # noqa: F401
