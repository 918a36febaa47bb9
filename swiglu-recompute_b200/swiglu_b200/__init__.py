"""B200-native (sm_100a) kernels of the SwiGLU-MLP recompute hot path.

The drop-in modules next to this package (`swiglu_recompute`, `fused_forward`,
`fused_forward_packed`, `fused_forward_packed_canon`) keep the reference
project's Python API and call into `libswiglu_b200.so` through `ops`.
"""
from . import ops  # noqa: F401
from ._lib import SwigluError, header_symbols, load  # noqa: F401
from .build import LIB_PATH, build  # noqa: F401
