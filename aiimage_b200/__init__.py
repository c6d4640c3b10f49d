"""aiimage_b200: B200 (sm_100a) backend for the Aexis quantized-decoder hot path.

The compute lives in libaexis_cuda.so (C ABI, include/aexis_cuda.h); this
package is its host-side binding: AexisOps (the reference's operator surface),
DecoderSession (its greedy decode loop) and the synthetic inputs used to
measure it.
"""
from . import errors  # noqa: F401
from .native import F16, F32  # noqa: F401

__all__ = ["errors", "F16", "F32"]
