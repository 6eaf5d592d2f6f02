"""Drop-in for the reference module ``kernels/fused_rmsnorm.py``.

``fused_add_rmsnorm(x, residual, weight, eps)`` -> (out, residual_out) with
out = rmsnorm(x + residual) * weight and residual_out = x + residual
(kernels/fused_rmsnorm.py:30-36), for bf16 activations and a bf16 weight (the
decode dtypes; fp32 math in a fixed order, see include/fp8gq.h).  The same
norm also runs as the prologue of the fused quant + GEMV:
``fused_add_rmsnorm_gemv_quant``.
"""
from .ops import RMS_EPS as EPS  # noqa: F401
from .ops import ShapeError, add_rmsnorm, fused_add_rmsnorm_gemv_quant  # noqa: F401


def fused_add_rmsnorm(x, residual, weight, eps=EPS):
    return add_rmsnorm(x, residual, weight, eps)


__all__ = ["fused_add_rmsnorm", "fused_add_rmsnorm_gemv_quant", "EPS", "ShapeError"]
