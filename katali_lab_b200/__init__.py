"""katali_lab_b200 — B200 (sm_100a) quantized expert hot path behind the katali_cuda C ABI.

The product is the shared library ``lib/libkatali_cuda.so`` (CUDA kernels and C
host code, built by ``build.py``) plus the dlopen shim
``lib/libkatali_cuda_loader.so``. This Python package only binds them
(``plugin.py``) for tests, the smoke test and the benchmark.
"""
from .plugin import (MOE_F32, MOE_NORM_TOPK, MOE_Q8_1, Q4_K, Q6_K, Q8_1, DenseModel,
                     ExpertCache, Gguf, HybridModel, KataliError, MoeLayer, Plugin, header_symbols)

__all__ = ["Plugin", "MoeLayer", "ExpertCache", "DenseModel", "HybridModel", "Gguf", "KataliError", "header_symbols", "Q4_K", "Q6_K", "Q8_1",
           "MOE_Q8_1", "MOE_F32", "MOE_NORM_TOPK"]
