"""Prepared launches: a linear's launch recorded once, issued many times.

A decode loop calls the same linears on the same buffers every step.  Most of
an eager call's host time goes to work that does not change between steps:
the argument checks, routing, tensor-map encoding, grid choice and the kernel
parameter block.  ``prepare_*`` does all of it once and returns a ``Plan``
(fp8gq_prepare_* in include/fp8gq.h); ``LaunchList(plans).run()`` then issues
every plan's kernels on the current stream with one C call
(fp8gq_launch_plans) and no other host work.  Launching a plan has the same
effect as the eager call it was prepared from.

A plan holds raw pointers: it keeps the tensors it was prepared with alive,
and must be prepared again when any of them is reallocated, or when
set_static_weights / set_tm_options change.  Plans that share a workspace
(all plans of one device and stream do) must not run concurrently.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib, ops


class Plan:
    """One prepared call (struct fp8gq_launch_plan) and the tensors it uses."""

    __slots__ = ("cplan", "keep", "out", "what")

    def __init__(self, what: str, keep, out=None):
        self.cplan = _lib.LaunchPlan()
        self.keep = keep
        self.out = out
        self.what = what

    def run(self, stream: int | None = None):
        LaunchList([self]).run(stream)
        return self.out


def _workspace(dev, M, N, K):
    lib = _lib.load()
    nbytes = ops._workspace_bytes(lib, dev, M, N, K)
    if not nbytes:
        return None, None, 0
    buf, ptr, n = ops._workspace_entry(dev, nbytes, ops._stream(dev))
    return buf, ptr, n


def prepare_fused_gemv_quant(x: torch.Tensor, Wq: torch.Tensor, Ws: torch.Tensor, out: torch.Tensor | None = None
                             ) -> Plan:
    """The plan of ``fused_gemv_quant(x, Wq, Ws, out=out)``; ``plan.out`` is the output."""
    ops._check_cuda(x, Wq, Ws)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise TypeError("x must be a 2-D bf16 tensor, contiguous along K")
    M, K = x.shape
    N, ldw, ldws = ops._check_weight_strides(Wq, Ws, K)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    buf, ws_ptr, ws_n = _workspace(x.device, M, N, K)
    plan = Plan("fp8gq_prepare_fused_gemv_quant", (x, Wq, Ws, out, buf), out)
    st = _lib.load().fp8gq_prepare_fused_gemv_quant(
        x.data_ptr(), x.stride(0), Wq.data_ptr(), ldw, Ws.data_ptr(), ldws, out.data_ptr(), out.stride(0),
        M, N, K, None, None, ws_ptr, ws_n, ctypes.byref(plan.cplan))
    _lib.check(st, plan.what)
    return plan


def prepare_fused_swiglu_q_gemm(gu: torch.Tensor, Wd: torch.Tensor, Ws: torch.Tensor,
                                out: torch.Tensor | None = None) -> Plan:
    """The plan of ``fused_swiglu_q_gemm(gu, Wd, Ws, out=out)``."""
    ops._check_cuda(gu, Wd, Ws)
    if gu.dtype != torch.bfloat16 or gu.dim() != 2 or gu.stride(1) != 1 or gu.shape[1] % 2:
        raise TypeError("gu must be a 2-D bf16 tensor [M, 2I], contiguous along its last dimension")
    M, I = gu.shape[0], gu.shape[1] // 2
    N, ldw, ldws = ops._check_weight_strides(Wd, Ws, I)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=gu.device)
    buf, ws_ptr, ws_n = _workspace(gu.device, M, N, I)
    plan = Plan("fp8gq_prepare_fused_swiglu_q_gemm", (gu, Wd, Ws, out, buf), out)
    st = _lib.load().fp8gq_prepare_fused_swiglu_q_gemm(
        gu.data_ptr(), gu.stride(0), Wd.data_ptr(), ldw, Ws.data_ptr(), ldws, out.data_ptr(), out.stride(0),
        M, N, I, None, None, ws_ptr, ws_n, ctypes.byref(plan.cplan))
    _lib.check(st, plan.what)
    return plan


def prepare_fused_add_rmsnorm_gemv_quant(x: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor,
                                         Wq: torch.Tensor, Ws: torch.Tensor, eps: float = ops.RMS_EPS, *,
                                         out: torch.Tensor | None = None,
                                         residual_out: torch.Tensor | None = None) -> Plan:
    """The plan of ``fused_add_rmsnorm_gemv_quant(x, residual, norm_weight, Wq, Ws, eps, out=,
    residual_out=)``; ``plan.out`` is the GEMV output."""
    M, K = ops._check_norm_inputs(x, residual, norm_weight)
    N, ldw, ldws = ops._check_weight_strides(Wq, Ws, K)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if residual_out is None:
        residual_out = torch.empty(M, K, dtype=torch.bfloat16, device=x.device)
    buf, ws_ptr, ws_n = _workspace(x.device, M, N, K)
    plan = Plan("fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant",
                (x, residual, norm_weight, Wq, Ws, out, residual_out, buf), out)
    st = _lib.load().fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant(
        x.data_ptr(), 1, 0, x.stride(0), residual.data_ptr(), residual.stride(0), norm_weight.data_ptr(), float(eps),
        Wq.data_ptr(), ldw, Ws.data_ptr(), ldws, out.data_ptr(), out.stride(0), residual_out.data_ptr(),
        residual_out.stride(0), M, N, K, None, None, None, ws_ptr, ws_n, ctypes.byref(plan.cplan))
    _lib.check(st, plan.what)
    return plan


class LaunchList:
    """Plans copied into one contiguous array; ``run()`` issues all of them,
    in order, on the current stream (or ``stream``) with one C call."""

    def __init__(self, plans):
        plans = list(plans)
        self.plans = plans
        self.n = len(plans)
        self.arr = (_lib.LaunchPlan * max(self.n, 1))()
        size = ctypes.sizeof(_lib.LaunchPlan)
        for i, p in enumerate(plans):
            ctypes.memmove(ctypes.byref(self.arr, i * size), ctypes.byref(p.cplan), size)
        self.device = None
        for p in plans:
            for t in p.keep:
                if isinstance(t, torch.Tensor) and t.is_cuda:
                    self.device = t.device
                    break
            if self.device is not None:
                break
        self._fn = _lib.load().fp8gq_launch_plans

    def run(self, stream: int | None = None):
        if stream is None:
            stream = ops._stream(self.device if self.device is not None else torch.device("cuda"))
        st = self._fn(self.arr, self.n, stream)
        if st:
            _lib.check(st, "fp8gq_launch_plans")
