"""Python host side of the B200 decode hot path (ctypes over libijb200.so).

The CUDA library is the product; this package loads it, mirrors the
reference's runner interface (FastRunner / FastGPU in inferencer.cu) for tests
and benchmarks, and generates the synthetic GGUF-layout models.  There is no
fallback: if libijb200.so is missing, loading fails with an error.
"""
from .lib import load, build, LIB_PATH  # noqa: F401
