"""B200-native (sm_100a) decode path for the ERNIE text decoder of
RapidAI/RapidOCRvl's PaddleOCR-VL runtime.

Public surface (mirrors the reference's internal/model API for this path):
  Runtime, LoadOptions, GenerateOptions, GenerateResult   (runtime.py)
  config.load / gguf.GGUFFile / gguf.convert              (formats)
The CUDA kernels live in csrc/ and are reached through the C ABI in
include/ocrvl_cuda.h (libocrvl_cuda.so, built in-tree by build.py).
"""
from .runtime import GenerateOptions, GenerateResult, LoadOptions, Runtime  # noqa: F401

__all__ = ["Runtime", "LoadOptions", "GenerateOptions", "GenerateResult"]
