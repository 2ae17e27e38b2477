"""xwfes_b200 -- B200-native (sm_100a) GGUF dequant-matmul backend.

The CUDA kernels and the C ABI live in libftcuda.so (built in-tree by
``python -m xwfes_b200.build``; interface in include/ftc.h).  ``ftc`` is its
ctypes binding plus a Python mirror of the reference's ft::IBackend;
``formats`` and ``synth`` hold the GGUF block geometry and the seeded
synthetic inputs of the benchmark configurations.
"""
from . import formats, synth  # noqa: F401

__all__ = ["formats", "synth", "ftc"]
