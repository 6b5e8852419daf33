"""B200 (sm_100a) backend for laguna-raw's quantized projection hot path.

The compute lives in liblaguna_cuda.so (C ABI, include/laguna_cuda.h); this
package holds its ctypes binding (lc), the seeded synthetic GGUF block
generators (synth) and the host-side model driver (dflash).
"""
from . import lc, synth  # noqa: F401

__all__ = ["lc", "synth"]
