"""Stack runner: a list of block-FP8 linears run by one persistent launch
(fp8gq_stack_prepare / fp8gq_stack_run in include/fp8gq.h).

Each linear is the fused activation quant + block-scaled GEMM of
``fused_gemv_quant`` (kernels/fused_gemv_quant_tm.py:49-80) or, with
``swiglu=True``, of ``fused_swiglu_q_gemm`` (kernels/fused_swiglu_quant_gemv.py:26-67).
A linear's input may be the output of an earlier linear of the list; the
kernel orders them (see ``dependencies``).  A decoder that owns its decode
step -- e.g. one CUDA graph per step -- prepares the list once and calls
``run()`` every step: one launch instead of one per linear, with every SM's
weight stream running on into the next linear while that linear waits for its
input.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, ops

MAX_TOKENS = 16


@dataclass
class Linear:
    """One linear of the list.  x: bf16 [M, K] ([M, 2K] = [gate | up] with
    swiglu), w: float8_e4m3fn [N, K], ws: fp32 [N/128, K/128], out: bf16 [M, N]."""
    x: torch.Tensor
    w: torch.Tensor
    ws: torch.Tensor
    out: torch.Tensor
    swiglu: bool = False


def _struct(lin: Linear) -> _lib.StackLinear:
    x, w, ws, out = lin.x, lin.w, lin.ws, lin.out
    for t, name in ((x, "x"), (out, "out")):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
            raise TypeError(f"{name} must be a 2-D bf16 tensor, contiguous along its last dimension")
    if w.dtype != torch.float8_e4m3fn or w.dim() != 2 or w.stride(1) != 1:
        raise TypeError("w must be a 2-D float8_e4m3fn tensor, contiguous along K")
    if ws.dtype != torch.float32 or ws.dim() != 2 or ws.stride(1) != 1:
        raise TypeError("ws must be a 2-D fp32 tensor, contiguous along its last dimension")
    N, K = w.shape
    M = x.shape[0]
    if x.shape[1] != (2 * K if lin.swiglu else K):
        raise ops.ShapeError(f"x must be [M, {2 * K if lin.swiglu else K}], got {tuple(x.shape)}")
    if out.shape != (M, N):
        raise ops.ShapeError(f"out must be [{M}, {N}], got {tuple(out.shape)}")
    if N % ops.GROUP or K % ops.GROUP:
        raise ops.ShapeError("N and K must be multiples of 128")
    if ws.shape[0] < N // ops.GROUP or ws.shape[1] < K // ops.GROUP:
        raise ops.ShapeError(f"ws must be [{N // ops.GROUP}, {K // ops.GROUP}], got {tuple(ws.shape)}")
    s = _lib.StackLinear()
    s.x, s.ldx = x.data_ptr(), x.stride(0)
    s.w, s.ldw = w.data_ptr(), w.stride(0)
    s.ws, s.ldws = ws.data_ptr(), ws.stride(0)
    s.out, s.ldo = out.data_ptr(), out.stride(0)
    s.N, s.K = N, K
    s.swiglu = 1 if lin.swiglu else 0
    s.reserved = 0
    return s


def _array(linears):
    if not linears:
        raise ValueError("the list is empty")
    M = linears[0].x.shape[0]
    if any(lin.x.shape[0] != M for lin in linears):
        raise ops.ShapeError("every linear of the list must have the same number of tokens M")
    if not 1 <= M <= MAX_TOKENS:
        raise ops.ShapeError(f"the stack runner takes 1 .. {MAX_TOKENS} tokens, got M = {M}")
    arr = (_lib.StackLinear * len(linears))(*[_struct(lin) for lin in linears])
    return arr, M


def dependencies(linears) -> list:
    """For each linear, the index of the earlier linear whose completion it
    waits for (-1: none) -- the latest one whose output overlaps its input or
    whose input or output overlaps its output."""
    arr, M = _array(linears)
    dep = (ctypes.c_int * len(linears))()
    lib = _lib.load()
    _lib.check(lib.fp8gq_stack_dependencies(arr, len(linears), M, dep), "fp8gq_stack_dependencies")
    return list(dep)


class StackRunner:
    """A prepared list of linears; ``run()`` launches all of them at once on
    the current stream.  Holds references to every tensor of the list (the
    plan stores their addresses): prepare a new runner after reallocating any
    of them."""

    def __init__(self, linears):
        linears = list(linears)
        ops._check_cuda(*[t for lin in linears for t in (lin.x, lin.w, lin.ws, lin.out)])
        dev = linears[0].x.device
        if any(t.device != dev for lin in linears for t in (lin.x, lin.w, lin.ws, lin.out)):
            raise ValueError("every tensor of the list must be on the same device")
        arr, M = _array(linears)
        self.linears = linears
        self.device = dev
        self.M = M
        lib = _lib.load()
        with torch.cuda.device(dev):
            nbytes = lib.fp8gq_stack_plan_bytes(len(linears), M)
            if nbytes == 0:
                raise _lib.Fp8gqError(6, "fp8gq_stack_plan_bytes")
            self.plan_mem = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            self.plan = _lib.StackPlan()
            _lib.check(lib.fp8gq_stack_prepare(arr, len(linears), M, self.plan_mem.data_ptr(), nbytes,
                                               ctypes.byref(self.plan), ops._stream(dev)), "fp8gq_stack_prepare")
        self._lib = lib

    @property
    def dependencies(self) -> list:
        return dependencies(self.linears)

    def run(self) -> None:
        """Every linear of the list, in order: one kernel launch on the
        current stream (capturable in a CUDA graph)."""
        _lib.check(self._lib.fp8gq_stack_run(ctypes.byref(self.plan), ops._stream(self.device)), "fp8gq_stack_run")
