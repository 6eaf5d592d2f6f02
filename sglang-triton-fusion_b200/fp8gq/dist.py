"""N-sharding of a block-FP8 linear across ranks (one process per GPU).

The output columns of a linear are independent, so rank r of `world` holds
rows [r*N/world, (r+1)*N/world) of the weight (whole 128-row blocks, so the
block scales split with it), runs the fused op on that slice and the bf16
slices are gathered on every rank.  The activation is replicated; every rank
quantises it itself.

Two ways to gather:
  * all_gather_columns / gathered_linear: the op, then an all-gather (NCCL on
    GPUs, gloo on CPU);
  * PeerGather: the kernel itself stores its slice into every rank's output
    buffer over NVLink (peer memory mapped with CUDA IPC) and raises a flag;
    the next gathered call waits for the flags inside its kernel.

Paired tensor parallelism (no gather between two linears): a column-parallel
linear (rows sharded as above; shard_gate_up keeps each rank's gate and up rows
together) leaves its slice on its rank, where it is the input of a row-parallel
linear (shard_cols: the K columns sharded) whose output is a partial sum.
PeerGather.linear_partial stores that partial into every rank's slab of a
[world, M, N] buffer, and PeerGather.reduce_norm_linear -- the next
column-parallel linear -- adds the slabs in rank order in its add + RMSNorm
prologue after waiting for every rank.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib, ops


def shard_rows(Wq: torch.Tensor, Ws: torch.Tensor, rank: int, world: int):
    """Rank `rank`'s slice of a weight [N, K] and its block scales [N/128, K/128]."""
    N = Wq.shape[0]
    nb = N // ops.GROUP
    if N % ops.GROUP or nb % world:
        raise ops.ShapeError(f"N/128 = {nb} row blocks do not split evenly over {world} ranks")
    per = nb // world
    return (Wq[rank * per * ops.GROUP:(rank + 1) * per * ops.GROUP],
            Ws[rank * per:(rank + 1) * per])


def shard_cols(Wq: torch.Tensor, Ws: torch.Tensor, rank: int, world: int):
    """Rank `rank`'s K slice of a weight [N, K] (columns, whole 128-column
    blocks) and of its block scales [N/128, K/128]: the row-parallel half of a
    pair, whose output is a partial sum over the slice."""
    K = Wq.shape[1]
    kb = K // ops.GROUP
    if K % ops.GROUP or kb % world:
        raise ops.ShapeError(f"K/128 = {kb} column blocks do not split evenly over {world} ranks")
    per = kb // world
    return (Wq[:, rank * per * ops.GROUP:(rank + 1) * per * ops.GROUP],
            Ws[:, rank * per:(rank + 1) * per])


def shard_gate_up(Wq: torch.Tensor, Ws: torch.Tensor, rank: int, world: int):
    """Rank `rank`'s rows of a merged [gate; up] weight [2I, K]: its slice of
    the gate rows followed by the same slice of the up rows (contiguous copies),
    so that its output is the [gate | up] input of a SwiGLU over its I/world
    intermediate columns."""
    I2 = Wq.shape[0]
    if I2 % 2:
        raise ops.ShapeError("the merged gate/up weight needs an even row count")
    I = I2 // 2
    gq, gs = shard_rows(Wq[:I], Ws[:I // ops.GROUP], rank, world)
    uq, us = shard_rows(Wq[I:], Ws[I // ops.GROUP:], rank, world)
    return torch.cat([gq, uq]).contiguous(), torch.cat([gs, us]).contiguous()


def all_gather_columns(shard: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """[M, Nr] per rank -> [M, world * Nr] with rank r's columns at r * Nr."""
    world = dist.get_world_size(group)
    M, Nr = shard.shape
    shard = shard.contiguous()
    gathered = torch.empty(world, M, Nr, dtype=shard.dtype, device=shard.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered.view(-1), shard.view(-1), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), shard, group=group)
    if M == 1 and out is None:
        return gathered.view(1, world * Nr)
    res = gathered.permute(1, 0, 2).reshape(M, world * Nr)
    if out is not None:
        out.copy_(res)
        return out
    return res


def gathered_linear(x: torch.Tensor, Wq_shard: torch.Tensor, Ws_shard: torch.Tensor, group=None,
                    op=None) -> torch.Tensor:
    """fused_gemv_quant on this rank's rows, then the all-gather: the full
    (M, N) output on every rank.  `op` defaults to fp8gq.fused_gemv_quant."""
    op = op or ops.fused_gemv_quant
    return all_gather_columns(op(x, Wq_shard, Ws_shard), group=group)


def untag(words: torch.Tensor) -> torch.Tensor:
    """The bf16 values of tagged words [M, N/2] (int64) as [M, N] (a copy)."""
    lo = words.contiguous().view(torch.int32)[..., 0::2].contiguous()
    return lo.view(torch.bfloat16).reshape(*words.shape[:-1], 2 * words.shape[-1])


def tags(words: torch.Tensor) -> torch.Tensor:
    """The sequence numbers of tagged words [M, N/2] (int64), as int64."""
    return (words >> 32) & 0xFFFFFFFF


class PeerGather:
    """Gathered linears over peer memory (fp8gq_fused_gemv_quant_gather).

    ``buffer`` is this rank's storage for full outputs: the same size, dtype
    bf16, on every rank.  It and a small flag array are mapped into every
    other rank (CUDA IPC, exchanged through ``group``).  ``linear`` writes the
    output of this rank's weight rows into columns ``col0 ..`` of ``out`` -- a
    [M, N] view into ``buffer`` -- on every rank at once.  Every rank must make
    the same sequence of ``linear`` calls.  ``wait()`` enqueues a wait for the
    last call's slices from every rank (before anything else reads ``out``).

    ``tagged=True`` selects tagged words (the fp8gq_gather ``tagged`` field):
    ``buffer`` is then int64, and an output [M, N] is a [M, N/2] view of it
    whose word i holds columns 2i, 2i + 1 and the sequence number of the call
    that wrote it.  No fence and no flag sits between a producer and its
    consumer: a call with ``wait_input`` takes such a view as ``x`` -- the
    output of the last call -- and its kernel polls the words it reads.
    ``decode(out, dst)`` waits for a tagged output and writes it as bf16.
    ``untag`` / ``tags`` read words on the host side.
    """

    def __init__(self, buffer: torch.Tensor, group=None, tagged: bool = False):
        want = torch.int64 if tagged else torch.bfloat16
        if buffer.dtype != want or not buffer.is_cuda or not buffer.is_contiguous():
            raise TypeError(f"buffer must be a contiguous CUDA {str(want).split('.')[-1]} tensor")
        self.tagged = bool(tagged)
        self.lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 2 <= self.world <= _lib.MAX_GATHER_RANKS:
            raise ValueError(f"PeerGather needs 2..{_lib.MAX_GATHER_RANKS} ranks, got {self.world}")
        self.buffer = buffer
        dev = buffer.device
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=dev)
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)        # counter, seq
        mine = (self._handle(buffer.data_ptr()), self._handle(self.flags.data_ptr()))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self._bases = []
        self.buf_ptrs, self.flag_ptrs = [], []
        for r, (hb, hf) in enumerate(allh):
            if r == self.rank:
                self.buf_ptrs.append(buffer.data_ptr())
                self.flag_ptrs.append(self.flags.data_ptr())
            else:
                self.buf_ptrs.append(self._open(hb))
                self.flag_ptrs.append(self._open(hf))
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def _handle(self, ptr):
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _lib.check(self.lib.fp8gq_ipc_get(ptr, h, ctypes.byref(off)), "fp8gq_ipc_get")
        return bytes(h.raw), int(off.value)

    def _open(self, hoff):
        h, off = hoff
        base, ptr = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(self.lib.fp8gq_ipc_open(ctypes.create_string_buffer(h, 64), off, ctypes.byref(base),
                                           ctypes.byref(ptr)), "fp8gq_ipc_open")
        self._bases.append(base.value)
        return ptr.value

    def descriptor(self, out: torch.Tensor, col0: int, wait_input: bool) -> "_lib.Gather":
        """The struct fp8gq_gather for output view ``out`` of ``buffer``
        (tagged: a word view; ldo and col0 count elements, two per word)."""
        es = out.element_size()
        off = out.data_ptr() - self.buffer.data_ptr()
        if (out.dtype != self.buffer.dtype or off < 0 or off + out.numel() * es > self.buffer.numel() * es
                or out.stride(1) != 1):
            raise ValueError("out must be a row-major view into the PeerGather buffer")
        g = _lib.Gather()
        for r in range(self.world):
            g.out[r] = self.buf_ptrs[r] + off
            g.flags[r] = self.flag_ptrs[r]
        g.counter = self.state.data_ptr()
        g.seq = self.state.data_ptr() + 4
        g.ldo = out.stride(0) * (2 if self.tagged else 1)
        g.col0 = col0
        g.world = self.world
        g.rank = self.rank
        g.wait_input = 1 if wait_input else 0
        g.tagged = 1 if self.tagged else 0
        return g

    def _cols(self, out: torch.Tensor) -> int:
        """Columns (elements) of an output view."""
        return out.shape[1] * (2 if self.tagged else 1)

    def _x_args(self, x: torch.Tensor, wait_input: bool):
        """(pointer, row stride in elements, K) of an input: tagged words when
        a tagged call waits for it, bf16 otherwise."""
        if self.tagged and wait_input:
            if x.dtype != torch.int64 or x.dim() != 2 or x.stride(1) != 1:
                raise TypeError("a tagged call that waits for its input takes a 2-D int64 word view")
            return x.data_ptr(), 2 * x.stride(0), 2 * x.shape[1]
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
            raise TypeError("x must be a 2-D bf16 tensor, contiguous along K")
        return x.data_ptr(), x.stride(0), x.shape[1]

    def linear(self, x: torch.Tensor, Wq_shard: torch.Tensor, Ws_shard: torch.Tensor, out: torch.Tensor,
               wait_input: bool = True, desc=None):
        """out[:, rank*Nr:(rank+1)*Nr] = fused_gemv_quant(x, Wq_shard, Ws_shard) on every rank."""
        return self._gathered(False, x, Wq_shard, Ws_shard, out, wait_input, desc)

    def swiglu_linear(self, gu: torch.Tensor, Wq_shard: torch.Tensor, Ws_shard: torch.Tensor, out: torch.Tensor,
                      wait_input: bool = True, desc=None):
        """out[:, rank*Nr:(rank+1)*Nr] = fused_swiglu_q_gemm(gu, Wq_shard, Ws_shard) on every rank
        (gu the full [gate | up] row, e.g. a gathered gate_up output)."""
        return self._gathered(True, gu, Wq_shard, Ws_shard, out, wait_input, desc)

    def _gathered(self, swiglu, x, Wq_shard, Ws_shard, out, wait_input, desc, plan=None):
        wait_input = bool(desc.wait_input) if desc is not None else wait_input
        xp, ldx, cols = self._x_args(x, wait_input)
        M = x.shape[0]
        if swiglu and cols % 2:
            raise ops.ShapeError("gu must hold [gate | up]: an even number of columns")
        K = cols // 2 if swiglu else cols
        Nr, ldw, ldws = ops._check_weight_strides(Wq_shard, Ws_shard, K)
        if out.shape[0] != M or self._cols(out) != Nr * self.world:
            raise ops.ShapeError(f"out must hold [{M}, {Nr * self.world}], got {tuple(out.shape)}")
        g = desc if desc is not None else self.descriptor(out, self.rank * Nr, wait_input)
        dev = x.device
        stream = ops._stream(dev)
        nbytes = ops._workspace_bytes(self.lib, dev, M, Nr, K)
        buf, ws_ptr, ws_n = ops._workspace_entry(dev, nbytes, stream) if nbytes else (None, None, 0)
        base = "fused_swiglu_q_gemm_gather" if swiglu else "fused_gemv_quant_gather"
        if plan is None:
            name = "fp8gq_" + base
            st = getattr(self.lib, name)(xp, ldx, Wq_shard.data_ptr(), ldw, Ws_shard.data_ptr(), ldws, M, Nr, K,
                                         ctypes.byref(g), ws_ptr, ws_n, stream)
            _lib.check(st, name)
            return out
        from .prepared import Plan
        name = "fp8gq_prepare_" + base
        pl = Plan(name, (x, Wq_shard, Ws_shard, out, buf, g), out)
        st = getattr(self.lib, name)(xp, ldx, Wq_shard.data_ptr(), ldw, Ws_shard.data_ptr(), ldws, M, Nr, K,
                                     ctypes.byref(g), ws_ptr, ws_n, ctypes.byref(pl.cplan))
        _lib.check(st, name)
        return pl

    def partial_descriptor(self, slabs: torch.Tensor) -> "_lib.Gather":
        """The struct fp8gq_gather that stores this rank's [M, N] partial into
        slab `rank` of ``slabs`` -- a [world, M, N] view into ``buffer`` -- on
        every rank."""
        if slabs.dim() != 3 or slabs.shape[0] != self.world or not slabs.is_contiguous():
            raise ValueError("slabs must be a contiguous [world, M, N] view into the PeerGather buffer")
        g = self.descriptor(slabs[self.rank], 0, False)
        off = slabs.data_ptr() - self.buffer.data_ptr() + self.rank * slabs.stride(0) * 2
        for r in range(self.world):
            g.out[r] = self.buf_ptrs[r] + off
        return g

    def wait_descriptor(self) -> "_lib.Gather":
        """A descriptor that only waits for every rank's last publishing call."""
        g = _lib.Gather()
        for r in range(self.world):
            g.flags[r] = self.flag_ptrs[r]
        g.counter = self.state.data_ptr()
        g.seq = self.state.data_ptr() + 4
        g.ldo = 1
        g.world = self.world
        g.rank = self.rank
        g.wait_input = 1
        g.local_out = 1
        return g

    def linear_partial(self, x: torch.Tensor, Wq_cols: torch.Tensor, Ws_cols: torch.Tensor, slabs: torch.Tensor,
                       swiglu: bool = False, desc=None):
        """The row-parallel half of a pair: this rank's partial output
        x @ Wq_cols^T (K slice; with swiglu, x is this rank's [gate | up]
        slice) stored into slab `rank` of ``slabs`` on every rank."""
        M = x.shape[0]
        N, Kr = Wq_cols.shape
        if slabs.shape[1:] != (M, N):
            raise ops.ShapeError(f"slabs must be [{self.world}, {M}, {N}], got {tuple(slabs.shape)}")
        if swiglu:
            if x.shape[1] != 2 * Kr:
                raise ops.ShapeError(f"gu must be [M, {2 * Kr}], got {tuple(x.shape)}")
        elif x.shape[1] != Kr:
            raise ops.ShapeError(f"x must be [M, {Kr}], got {tuple(x.shape)}")
        _, ldw, ldws = ops._check_weight_strides(Wq_cols, Ws_cols, Kr)
        g = desc if desc is not None else self.partial_descriptor(slabs)
        dev = x.device
        stream = ops._stream(dev)
        nbytes = ops._workspace_bytes(self.lib, dev, M, N, Kr)
        ws_ptr, ws_n = ops._workspace_entry(dev, nbytes, stream)[1:] if nbytes else (None, 0)
        fn = self.lib.fp8gq_fused_swiglu_q_gemm_gather if swiglu else self.lib.fp8gq_fused_gemv_quant_gather
        st = fn(x.data_ptr(), x.stride(0), Wq_cols.data_ptr(), ldw, Ws_cols.data_ptr(), ldws, M, N, Kr,
                ctypes.byref(g), ws_ptr, ws_n, stream)
        _lib.check(st, "fp8gq_fused_swiglu_q_gemm_gather" if swiglu else "fp8gq_fused_gemv_quant_gather")
        return slabs

    def reduce_norm_linear(self, slabs: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor,
                           Wq_rows: torch.Tensor, Ws_rows: torch.Tensor, out: torch.Tensor,
                           residual_out: torch.Tensor, eps: float = ops.RMS_EPS, desc=None):
        """The next column-parallel linear: waits for every rank's partial,
        then out = GEMV(quant(rmsnorm(sum of slabs in rank order + residual)))
        on this rank's rows; residual_out = bf16(sum + residual)."""
        g = desc if desc is not None else self.wait_descriptor()
        return ops.fused_reduce_add_rmsnorm_gemv_quant(slabs, residual, norm_weight, Wq_rows, Ws_rows, eps,
                                                       out=out, residual_out=residual_out, wait=g)

    # ---- prepared launches (fp8gq.prepared): the same calls, recorded once
    def prepare_linear(self, x: torch.Tensor, Wq_shard: torch.Tensor, Ws_shard: torch.Tensor, out: torch.Tensor,
                       wait_input: bool = True, desc=None):
        """The plan of ``linear(x, Wq_shard, Ws_shard, out, wait_input)``."""
        return self._gathered(False, x, Wq_shard, Ws_shard, out, wait_input, desc, plan=True)

    def prepare_swiglu_linear(self, gu: torch.Tensor, Wq_shard: torch.Tensor, Ws_shard: torch.Tensor,
                              out: torch.Tensor, wait_input: bool = True, desc=None):
        """The plan of ``swiglu_linear(gu, Wq_shard, Ws_shard, out, wait_input)``."""
        return self._gathered(True, gu, Wq_shard, Ws_shard, out, wait_input, desc, plan=True)

    def prepare_linear_partial(self, x: torch.Tensor, Wq_cols: torch.Tensor, Ws_cols: torch.Tensor,
                               slabs: torch.Tensor, swiglu: bool = False, desc=None):
        """The plan of ``linear_partial(x, Wq_cols, Ws_cols, slabs, swiglu)``."""
        from .prepared import Plan
        M = x.shape[0]
        N, Kr = Wq_cols.shape
        if slabs.shape[1:] != (M, N):
            raise ops.ShapeError(f"slabs must be [{self.world}, {M}, {N}], got {tuple(slabs.shape)}")
        if x.shape[1] != (2 * Kr if swiglu else Kr):
            raise ops.ShapeError(f"input must be [M, {2 * Kr if swiglu else Kr}], got {tuple(x.shape)}")
        _, ldw, ldws = ops._check_weight_strides(Wq_cols, Ws_cols, Kr)
        g = desc if desc is not None else self.partial_descriptor(slabs)
        dev = x.device
        nbytes = ops._workspace_bytes(self.lib, dev, M, N, Kr)
        buf, ws_ptr, ws_n = ops._workspace_entry(dev, nbytes, ops._stream(dev)) if nbytes else (None, None, 0)
        name = "fp8gq_prepare_fused_swiglu_q_gemm_gather" if swiglu else "fp8gq_prepare_fused_gemv_quant_gather"
        plan = Plan(name, (x, Wq_cols, Ws_cols, slabs, buf, g), slabs)
        st = getattr(self.lib, name)(x.data_ptr(), x.stride(0), Wq_cols.data_ptr(), ldw, Ws_cols.data_ptr(), ldws,
                                     M, N, Kr, ctypes.byref(g), ws_ptr, ws_n, ctypes.byref(plan.cplan))
        _lib.check(st, name)
        return plan

    def prepare_reduce_norm_linear(self, slabs: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor,
                                   Wq_rows: torch.Tensor, Ws_rows: torch.Tensor, out: torch.Tensor,
                                   residual_out: torch.Tensor, eps: float = ops.RMS_EPS, desc=None):
        """The plan of ``reduce_norm_linear(...)``."""
        from .prepared import Plan
        if slabs.dim() != 3 or not 1 <= slabs.shape[0] <= _lib.MAX_GATHER_RANKS:
            raise ops.ShapeError("slabs must be [S, M, K] with 1 <= S <= 8")
        M, K = ops._check_norm_inputs(slabs[0], residual, norm_weight)
        N, ldw, ldws = ops._check_weight_strides(Wq_rows, Ws_rows, K)
        if out.shape != (M, N) or residual_out.shape != (M, K):
            raise ops.ShapeError("out must be [M, N] and residual_out [M, K]")
        g = desc if desc is not None else self.wait_descriptor()
        dev = slabs.device
        nbytes = ops._workspace_bytes(self.lib, dev, M, N, K)
        buf, ws_ptr, ws_n = ops._workspace_entry(dev, nbytes, ops._stream(dev)) if nbytes else (None, None, 0)
        name = "fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant"
        plan = Plan(name, (slabs, residual, norm_weight, Wq_rows, Ws_rows, out, residual_out, buf, g), out)
        st = self.lib.fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant(
            slabs.data_ptr(), slabs.shape[0], slabs.stride(0), slabs.stride(1), residual.data_ptr(), residual.stride(0),
            norm_weight.data_ptr(), float(eps), Wq_rows.data_ptr(), ldw, Ws_rows.data_ptr(), ldws, out.data_ptr(),
            out.stride(0), residual_out.data_ptr(), residual_out.stride(0), M, N, K, None, None, ctypes.byref(g),
            ws_ptr, ws_n, ctypes.byref(plan.cplan))
        _lib.check(st, name)
        return plan

    def decode(self, out: torch.Tensor, dst: torch.Tensor | None = None) -> torch.Tensor:
        """Tagged words: enqueue a kernel that waits until every word of the
        full output ``out`` (a word view, the last call's output) has arrived
        and writes its values into ``dst`` (bf16 [M, N], made if None)."""
        g, dst, M, N = self._decode_args(out, dst)
        _lib.check(self.lib.fp8gq_gather_decode(ctypes.byref(g), M, N, dst.data_ptr(), dst.stride(0),
                                                ops._stream(out.device)), "fp8gq_gather_decode")
        return dst

    def prepare_decode(self, out: torch.Tensor, dst: torch.Tensor | None = None):
        """The plan of ``decode(out, dst)``; ``plan.out`` is ``dst``."""
        from .prepared import Plan
        g, dst, M, N = self._decode_args(out, dst)
        plan = Plan("fp8gq_prepare_gather_decode", (out, dst, g), dst)
        _lib.check(self.lib.fp8gq_prepare_gather_decode(ctypes.byref(g), M, N, dst.data_ptr(), dst.stride(0),
                                                        ctypes.byref(plan.cplan)), plan.what)
        return plan

    def _decode_args(self, out, dst):
        if not self.tagged:
            raise ValueError("decode is for tagged words; use wait() with flags")
        M, N = out.shape[0], self._cols(out)
        if dst is None:
            dst = torch.empty(M, N, dtype=torch.bfloat16, device=out.device)
        if dst.dtype != torch.bfloat16 or tuple(dst.shape) != (M, N) or dst.stride(1) != 1:
            raise ops.ShapeError(f"dst must be a bf16 [{M}, {N}] tensor, contiguous along its rows")
        return self.descriptor(out, 0, True), dst, M, N

    def prepare_wait(self, out: torch.Tensor):
        """The plan of ``wait(out)``."""
        from .prepared import Plan
        if self.tagged:
            raise ValueError("tagged words are waited for by prepare_decode(out, dst)")
        g = self.descriptor(out, 0, True)
        plan = Plan("fp8gq_prepare_gather_wait", (out, g), out)
        _lib.check(self.lib.fp8gq_prepare_gather_wait(ctypes.byref(g), ctypes.byref(plan.cplan)), plan.what)
        return plan

    def wait(self, out: torch.Tensor):
        """Enqueue a wait for the last gathered call's slices from every rank."""
        if self.tagged:
            raise ValueError("tagged words are waited for by decode(out, dst)")
        g = self.descriptor(out, 0, True)
        _lib.check(self.lib.fp8gq_gather_wait(ctypes.byref(g), ops._stream(out.device)), "fp8gq_gather_wait")

    def close(self):
        torch.cuda.synchronize(self.buffer.device)
        dist.barrier(group=self.group)
        for b in self._bases:
            self.lib.fp8gq_ipc_close(b)
        self._bases = []
