"""Drop-in for the reference module ``kernels/fused_gemv_quant_tm.py``: the
module the sglang patch imports (patches/patch_fp8_fused_tail.py:20).

``fused_gemv_quant(x, Wq, Ws)`` keeps the reference's contract
(kernels/fused_gemv_quant_tm.py:83-102): x (M, K) bf16, Wq (N, K) e4m3,
Ws (N/128, K/128) fp32 -> (M, N) bf16; M == 1 runs the row kernel, M > 1 the
tile kernel (here on tcgen05 tensor cores); K, N not multiples of 128 raise
AssertionError (a ShapeError).
"""
from .ops import TM, ShapeError, fused_gemv_quant  # noqa: F401

__all__ = ["TM", "fused_gemv_quant", "ShapeError"]
