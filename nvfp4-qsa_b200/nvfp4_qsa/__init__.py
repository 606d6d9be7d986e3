"""NVFP4 paged KV cache + QSA sparse decode attention for B200 (sm_100a).

Drop-in for the reference package ``nvfp4_qsa`` (python/nvfp4_qsa/__init__.py):
the same top-level names, with every kernel a hand-written sm_100a CUDA kernel
behind the C ABI in include/nvfp4_qsa.h.  The native library is loaded lazily
on the first kernel call.
"""
from .codec import encode, decode, global_scale_for
from .cache import PackedCache

__version__ = "0.1.0"
__all__ = ["encode", "decode", "global_scale_for", "PackedCache"]
