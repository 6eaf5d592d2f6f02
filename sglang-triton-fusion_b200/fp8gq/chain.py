"""Chain runner: a decode step's M == 1 linears in one persistent launch.

fp8gq_chain_* (include/fp8gq.h).  Each linear is N-sharded across the ranks of
a tagged PeerGather (or runs whole on one GPU) and stores its rows as tagged
words into every rank's output; a linear whose input is an earlier linear's
output polls the words it reads, so the whole list runs as one cooperative
launch with no barrier between linears.  The math and its order are the row
kernel's (fp8gq_fused_gemv_quant_gather).

    runner = ChainRunner([
        Link(x=h, w=wq0, ws=ws0, out=o0),                     # bf16 step input
        Link(x=o0[:, :2048], w=wq1, ws=ws1, out=o1, src=0),   # first 4096 columns of o0
        ...])
    runner.run()                 # one launch per step
    y = runner.decode(o_last)    # bf16 result of the last linear

Outputs are int64 word views [1, N/2] (N the full width): views of the
PeerGather's buffer on several GPUs, any CUDA int64 tensors on one.  The
weights must not change between runs (they are read without waiting for
earlier work on the stream).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib, ops


@dataclass
class Link:
    """One linear of a chain: out = GEMV(quant(x)) on this rank's weight rows."""
    x: torch.Tensor              # bf16 [1, K] ([1, 2K] with swiglu) when src < 0, else a word view
    w: torch.Tensor              # e4m3 [N_shard, K]
    ws: torch.Tensor             # fp32 [N_shard / 128, K / 128]
    out: torch.Tensor            # int64 word view [1, N_full / 2]
    src: int = -1                # the earlier linear whose output x views
    swiglu: bool = False


class ChainRunner:
    """A prepared chain (fp8gq_chain_prepare); ``run()`` launches it."""

    def __init__(self, links, gather=None):
        self.lib = _lib.load()
        self.links = list(links)
        n = len(self.links)
        if n < 1:
            raise ValueError("a chain needs at least one linear")
        dev = self.links[0].w.device
        self.device = dev
        self.gather = gather
        if gather is not None:
            if not gather.tagged:
                raise ValueError("the chain runner needs a PeerGather with tagged=True")
            world, rank = gather.world, gather.rank
            flag_ptrs, state = gather.flag_ptrs, gather.state
        else:
            world, rank = 1, 0
            self.flags = torch.zeros(1, dtype=torch.int32, device=dev)
            self.state = torch.zeros(2, dtype=torch.int32, device=dev)      # counter, seq
            flag_ptrs, state = [self.flags.data_ptr()], self.state
        self.world, self.rank = world, rank
        table = (_lib.ChainLinear * n)()
        for i, lk in enumerate(self.links):
            t = table[i]
            if lk.out.dtype != torch.int64 or lk.out.dim() != 2 or lk.out.shape[0] != 1 or lk.out.stride(1) != 1:
                raise TypeError(f"link {i}: out must be an int64 word view [1, N/2]")
            if lk.src >= 0:
                if lk.x.dtype != torch.int64 or lk.x.dim() != 2 or lk.x.stride(1) != 1:
                    raise TypeError(f"link {i}: x must be a word view of linear {lk.src}'s output")
                cols = 2 * lk.x.shape[1]
            else:
                if lk.x.dtype != torch.bfloat16 or lk.x.dim() != 2 or lk.x.shape[0] != 1 or lk.x.stride(1) != 1:
                    raise TypeError(f"link {i}: x must be a bf16 [1, K] tensor")
                cols = lk.x.shape[1]
            K = cols // 2 if lk.swiglu else cols
            N, ldw, ldws = ops._check_weight_strides(lk.w, lk.ws, K)
            if 2 * lk.out.shape[1] != N * world:
                raise ops.ShapeError(f"link {i}: out holds {2 * lk.out.shape[1]} columns, expected {N * world}")
            t.x = lk.x.data_ptr()
            t.w = lk.w.data_ptr()
            t.ldw = ldw
            t.ws = lk.ws.data_ptr()
            t.ldws = ldws
            t.N = N
            t.K = K
            t.src = lk.src
            t.swiglu = 1 if lk.swiglu else 0
            t.col0 = rank * N
            t.reserved = 0
            for r in range(world):
                if gather is not None:
                    t.out[r] = gather.buf_ptrs[r] + (lk.out.data_ptr() - gather.buffer.data_ptr())
                else:
                    t.out[r] = lk.out.data_ptr()
        self.table = table
        g = _lib.Gather()
        for q in range(world):
            g.flags[q] = flag_ptrs[q]
        g.counter = state.data_ptr()
        g.seq = state.data_ptr() + 4
        g.world = world
        g.rank = rank
        g.tagged = 1
        self._g = g
        nbytes = self.lib.fp8gq_chain_plan_bytes(n)
        self.mem = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
        base = (self.mem.data_ptr() + 255) // 256 * 256
        self.plan = _lib.ChainPlan()
        _lib.check(self.lib.fp8gq_chain_prepare(table, n, ctypes.byref(g), base, nbytes, ctypes.byref(self.plan)),
                   "fp8gq_chain_prepare")

    def run(self, stream: int | None = None):
        """Launch the chain on the current stream (or ``stream``)."""
        if stream is None:
            stream = ops._stream(self.device)
        _lib.check(self.lib.fp8gq_chain_run(ctypes.byref(self.plan), stream), "fp8gq_chain_run")

    def decode(self, out: torch.Tensor, dst: torch.Tensor | None = None) -> torch.Tensor:
        """Wait for every word of ``out`` (the last linear's output) and write it as bf16."""
        if self.gather is not None:
            return self.gather.decode(out, dst)
        M, N = out.shape[0], 2 * out.shape[1]
        if dst is None:
            dst = torch.empty(M, N, dtype=torch.bfloat16, device=out.device)
        g = _lib.Gather()
        g.out[0] = out.data_ptr()
        g.flags[0] = self.flags.data_ptr()
        g.counter = self.state.data_ptr()
        g.seq = self.state.data_ptr() + 4
        g.ldo = 2 * out.stride(0)
        g.world = 1
        g.rank = 0
        g.wait_input = 1
        g.tagged = 1
        _lib.check(self.lib.fp8gq_gather_decode(ctypes.byref(g), M, N, dst.data_ptr(), dst.stride(0),
                                                ops._stream(out.device)), "fp8gq_gather_decode")
        return dst
