"""Module path kept from the reference package (``nvfp4_qsa.oracle``).

The reference names its CPU codec module ``oracle``; callers import
``from nvfp4_qsa.oracle import encode, decode``.  Here the same names resolve
to the GPU codec in ``nvfp4_qsa.codec`` (csrc/codec.cu).  This module is not
the test oracle (that is the top-level ``oracle/`` directory, which the
package never imports).
"""
from .codec import E2M1_GRID, E2M1_MAX, E4M3_MAX, GROUP, decode, encode, global_scale_for, quant_dequant

__all__ = ["E2M1_GRID", "E2M1_MAX", "E4M3_MAX", "GROUP", "encode", "decode", "global_scale_for", "quant_dequant"]
