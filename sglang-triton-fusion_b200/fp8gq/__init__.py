"""fp8gq: fused FP8 (e4m3) activation group-quant + block-scaled GEMV for
NVIDIA B200 (sm_100a), behind the drop-in surface of the sglang patch
``patches/patch_fp8_fused_tail.py`` of wafik/sglang-triton-fusion.

Entry points:
  fused_gemv_quant(x, Wq, Ws)      M == 1 row kernel / M > 1 tcgen05 tile kernel
  fused_swiglu_q_gemm(gu, Wd, Ws)  SwiGLU + quant + down_proj GEMV
  group_quant(x), swiglu_group_quant(gu)   the activation quant alone
  fused_swiglu(g, u), fused_swiglu_quant(g, u)   stand-alone SwiGLU writers (large M)
  add_rmsnorm(x, r, w), fused_add_rmsnorm_gemv_quant(x, r, w, Wq, Ws)   add + RMSNorm (prologue)
  fused_reduce_add_rmsnorm_gemv_quant(partials, r, w, Wq, Ws)          + the sum of K-sharded partials
  StackRunner([Linear(x, Wq, Ws, out, swiglu)...])   a list of linears in one persistent launch
  prepare_fused_gemv_quant(...), LaunchList(plans).run()   calls recorded once, launched with no host work
  patch_fp8_fused_tail             the sglang linear wrappers and install()
The C ABI is include/fp8gq.h (libfp8gq.so next to this file).
"""
from ._lib import (TM_PREQUANT_ACTIVATIONS, TM_RESIDENT_ACTIVATIONS, TM_STREAM_ACTIVATIONS,  # noqa: F401
                   TM_WORKSPACE_SPLITK, Fp8gqError, device_error, load, set_static_weights, set_tm_options,
                   set_wait_limit_ns)
from .ops import (GROUP, TM, ShapeError, add_rmsnorm, fused_add_rmsnorm_gemv_quant,  # noqa: F401
                  fused_reduce_add_rmsnorm_gemv_quant,
                  fused_gemv_quant, fused_swiglu, fused_swiglu_q_gemm, fused_swiglu_quant, group_quant,
                  swiglu_group_quant, workspace)
from .prepared import (LaunchList, Plan, prepare_fused_add_rmsnorm_gemv_quant, prepare_fused_gemv_quant,  # noqa: F401
                       prepare_fused_swiglu_q_gemm)
from .stack import Linear, StackRunner  # noqa: F401
from .chain import ChainRunner, Link  # noqa: F401

__all__ = ["Fp8gqError", "ShapeError", "GROUP", "TM", "fused_gemv_quant", "fused_swiglu_q_gemm",
           "fused_swiglu", "fused_swiglu_quant", "add_rmsnorm", "fused_add_rmsnorm_gemv_quant",
           "fused_reduce_add_rmsnorm_gemv_quant",
           "group_quant", "swiglu_group_quant", "workspace", "load", "device_error", "set_static_weights",
           "set_tm_options", "set_wait_limit_ns", "TM_STREAM_ACTIVATIONS", "TM_WORKSPACE_SPLITK",
           "TM_PREQUANT_ACTIVATIONS", "TM_RESIDENT_ACTIVATIONS", "Linear", "StackRunner",
           "LaunchList", "Plan", "prepare_fused_gemv_quant", "prepare_fused_swiglu_q_gemm",
           "prepare_fused_add_rmsnorm_gemv_quant"]
