"""quantfun2_b200: B200-native (sm_100a) kernels for quantfun2's DiT inference hot path.

Drop-in ops for the reference's seams:
  * kernel seam  (src/kernels/__init__.py)      -> quantfun2_b200.kernels
  * attention    (ATTN switch, sageattention)   -> quantfun2_b200.attention

All compute runs in libqf2b200.so (hand-written CUDA for sm_100a, C ABI in
include/qf2b200.h).  Build it with ``python quantfun2_b200/build.py``.
"""
from ._lib import QF2Error, LIB_PATH, load  # noqa: F401

__version__ = "0.1.0"
