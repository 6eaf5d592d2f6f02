"""Drop-in for the reference module ``kernels/fused_swiglu_fp8.py``: the
stand-alone SwiGLU writers used where M is too large for the fused GEMV path.

``fused_swiglu(gate, up)`` -> bf16 silu(gate) * up (kernels/fused_swiglu_fp8.py:48-53);
``fused_swiglu_quant(gate, up)`` -> (e4m3 q, fp32 scale) with that module's
formula, scale = max(amax / 448, 1e-30), q = e4m3(clamp(y / scale, +-448))
(kernels/fused_swiglu_fp8.py:56-63).  GROUP and QMAX are the module's constants.
"""
from .ops import GROUP, ShapeError, fused_swiglu, fused_swiglu_quant  # noqa: F401

QMAX = 448.0

__all__ = ["fused_swiglu", "fused_swiglu_quant", "GROUP", "QMAX", "ShapeError"]
