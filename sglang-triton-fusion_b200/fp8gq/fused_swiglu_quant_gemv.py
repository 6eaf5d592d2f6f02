"""Drop-in for the reference module ``kernels/fused_swiglu_quant_gemv.py``.

``fused_swiglu_q_gemm(gu, Wd, Ws)`` keeps the reference's contract
(kernels/fused_swiglu_quant_gemv.py:54-67): gu (M, 2I) bf16 = [gate | up],
Wd (N, I) e4m3, Ws (N/128, I/128) fp32 -> (M, N) bf16 of
GEMV(quant(silu(gate) * up)).
"""
from .ops import ShapeError, fused_swiglu_q_gemm  # noqa: F401

__all__ = ["fused_swiglu_q_gemm", "ShapeError"]
