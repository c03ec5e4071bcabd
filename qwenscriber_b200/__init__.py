"""qwenscriber_b200: the sm_100a (B200) backend of Qwenscriber's decoder token loop.

The compute lives in `libqwenscriber_cuda.so` (hand-written CUDA for sm_100a
behind the C ABI of include/qwenscriber_cuda.h); this package holds its Python
host binding, the 160-byte model configuration, the host-side quantizer and
the seeded synthetic models the benchmarks run.
"""

from . import config, quant, synthetic
from .runtime import CudaModel, QwcError, lib

__all__ = ["CudaModel", "QwcError", "lib", "config", "quant", "synthetic"]
