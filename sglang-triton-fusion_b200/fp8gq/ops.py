"""torch-tensor front end of libfp8gq: checks dtypes and layouts, allocates
the output from torch's caching allocator (as the reference wrapper does,
kernels/fused_gemv_quant_tm.py:89) and launches on torch's current stream.

Every op runs the CUDA kernels; there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib

GROUP = 128
TM = 16  # largest M routed to the fused kernels by the patch layer


class ShapeError(AssertionError, ValueError):
    """Shape the fused path does not take (the reference asserts the same:
    kernels/fused_gemv_quant_tm.py:87)."""


def _ptr(t):
    return None if t is None else t.data_ptr()


try:
    _raw_stream = torch._C._cuda_getCurrentRawStream   # the current stream's handle, without a Stream object
except AttributeError:                                  # pragma: no cover
    _raw_stream = None


def _stream(device) -> int:
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


_workspaces: dict = {}
_ws_bytes: dict = {}


def _workspace_bytes(lib, device, M, N, K, tile_only=False) -> int:
    """fp8gq_workspace_bytes, remembered per (device, shape)."""
    key = (device.index, M, N, K, tile_only)
    n = _ws_bytes.get(key)
    if n is None:
        n = lib.fp8gq_workspace_bytes(max(M, 2) if tile_only else M, N, K)
        _ws_bytes[key] = n
    return n


def workspace(device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
    """Zero-filled scratch kept per (device, stream).  The kernels leave it
    zero-filled when they finish, so it is allocated and cleared once; grow it
    (and warm every shape up) before capturing a CUDA graph."""
    if stream is None:
        stream = _stream(device)
    return _workspace_entry(device, nbytes, stream)[0]


def _workspace_entry(device: torch.device, nbytes: int, stream: int):
    """(tensor, address, bytes) of the scratch of (device, stream), at least
    nbytes; the address and size are kept so that a call needs no tensor
    method to pass them."""
    key = (device.index, stream)
    ent = _workspaces.get(key)
    if ent is None or ent[2] < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        ent = (buf, buf.data_ptr(), buf.numel())
        _workspaces[key] = ent
    return ent


def _check_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("fp8gq ops take CUDA tensors only (there is no CPU path)")


def _check_weight(Wq: torch.Tensor, Ws: torch.Tensor, K: int):
    """Checks a weight and its block scales against K; returns N."""
    return _check_weight_strides(Wq, Ws, K)[0]


def _check_weight_strides(Wq: torch.Tensor, Ws: torch.Tensor, K: int):
    """_check_weight, also returning the row strides: (N, ldw, ldws)."""
    if Wq.dtype != torch.float8_e4m3fn:
        raise TypeError(f"weight must be float8_e4m3fn, got {Wq.dtype}")
    if Ws.dtype != torch.float32:
        raise TypeError(f"weight_scale must be float32, got {Ws.dtype}")
    N, Kw = Wq.shape
    if Kw != K:
        raise ShapeError(f"weight has K={Kw}, activation has K={K}")
    if K % GROUP or N % GROUP:
        raise ShapeError("K and N must be multiples of 128")
    ws_t = Wq.stride()
    ss_t = Ws.stride()
    if ws_t[1] != 1 or ss_t[1] != 1:
        raise ValueError("weight and weight_scale must be contiguous along K")
    if Ws.shape != (N // GROUP, K // GROUP):
        raise ShapeError(f"weight_scale must be [{N // GROUP}, {K // GROUP}], got {tuple(Ws.shape)}")
    return N, ws_t[0], ss_t[0]


def _quant_out(M, K, device, want):
    if not want:
        return None, None
    return (torch.empty(M, K, dtype=torch.uint8, device=device),
            torch.empty(M, K // GROUP, dtype=torch.float32, device=device))


def fused_gemv_quant(x: torch.Tensor, Wq: torch.Tensor, Ws: torch.Tensor, *, out=None,
                     return_quant: bool = False, kernel: str = "auto"):
    """x: (M, K) bf16; Wq: (N, K) e4m3; Ws: (N/128, K/128) fp32 -> (M, N) bf16.

    Same contract as fused_gemv_quant (kernels/fused_gemv_quant_tm.py:83-102):
    M == 1 runs the row kernel, M > 1 the tensor-core tile kernel.
    ``kernel`` = "row" or "tm" forces one of them; ``return_quant`` also
    returns the quantised activation bytes (uint8 e4m3 codes) and scales that
    the kernel computed internally."""
    _check_cuda(x, Wq, Ws)
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("x must be a 2-D bf16 tensor")
    M, K = x.shape
    N, ldw, ldws = _check_weight_strides(Wq, Ws, K)
    xs = x.stride()
    if xs[1] != 1:
        raise ValueError("x must be contiguous along K")
    dev = x.device
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    xq, sx = _quant_out(M, K, dev, return_quant)
    lib = _lib.load()
    stream = _stream(dev)
    if kernel == "row":
        if M != 1:
            raise ShapeError("the row kernel takes M == 1")
        st = lib.fp8gq_gemv_quant_row(x.data_ptr(), Wq.data_ptr(), ldw, Ws.data_ptr(), ldws, out.data_ptr(),
                                      N, K, _ptr(xq), _ptr(sx), stream)
        _lib.check(st, "fp8gq_gemv_quant_row")
    else:
        if kernel not in ("auto", "tm"):
            raise ValueError(f"unknown kernel {kernel!r}")
        nbytes = _workspace_bytes(lib, dev, M, N, K, tile_only=kernel != "auto")
        ws_ptr, ws_n = _workspace_entry(dev, nbytes, stream)[1:] if nbytes else (None, 0)
        fn = lib.fp8gq_fused_gemv_quant if kernel == "auto" else lib.fp8gq_gemv_quant_tm
        st = fn(x.data_ptr(), xs[0], Wq.data_ptr(), ldw, Ws.data_ptr(), ldws, out.data_ptr(), out.stride(0),
                M, N, K, _ptr(xq), _ptr(sx), ws_ptr, ws_n, stream)
        _lib.check(st, fn.__name__)
    return (out, xq, sx) if return_quant else out


def fused_swiglu_q_gemm(gu: torch.Tensor, Wd: torch.Tensor, Ws: torch.Tensor, *, out=None,
                        return_quant: bool = False):
    """gu: (M, 2I) bf16 gate_up output ([gate | up]); Wd: (N, I) e4m3;
    Ws: (N/128, I/128) fp32 -> (M, N) bf16
    (kernels/fused_swiglu_quant_gemv.py:54-67)."""
    _check_cuda(gu, Wd, Ws)
    if gu.dtype != torch.bfloat16 or gu.dim() != 2:
        raise TypeError("gu must be a 2-D bf16 tensor")
    M, two_i = gu.shape
    if two_i % 2:
        raise ShapeError("gu must have an even number of columns ([gate | up])")
    I = two_i // 2
    N = _check_weight(Wd, Ws, I)
    if gu.stride(1) != 1:
        raise ValueError("gu must be contiguous along its last dimension")
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=gu.device)
    xq, sx = _quant_out(M, I, gu.device, return_quant)
    lib = _lib.load()
    nbytes = _workspace_bytes(lib, gu.device, M, N, I)
    ws_buf = workspace(gu.device, nbytes) if nbytes else None
    st = lib.fp8gq_fused_swiglu_q_gemm(_ptr(gu), gu.stride(0), _ptr(Wd), Wd.stride(0), _ptr(Ws), Ws.stride(0),
                                       _ptr(out), out.stride(0), M, N, I, _ptr(xq), _ptr(sx), _ptr(ws_buf),
                                       0 if ws_buf is None else ws_buf.numel(), _stream(gu.device))
    _lib.check(st, "fp8gq_fused_swiglu_q_gemm")
    return (out, xq, sx) if return_quant else out


def group_quant(x: torch.Tensor):
    """x: (M, K) bf16 -> (xq uint8 e4m3 codes (M, K), sx fp32 (M, K/128))."""
    _check_cuda(x)
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise TypeError("x must be a 2-D bf16 tensor, contiguous along K")
    M, K = x.shape
    xq, sx = _quant_out(M, K, x.device, True)
    lib = _lib.load()
    _lib.check(lib.fp8gq_group_quant(_ptr(x), x.stride(0), M, K, _ptr(xq), _ptr(sx), _stream(x.device)),
               "fp8gq_group_quant")
    return xq, sx


def swiglu_group_quant(gu: torch.Tensor):
    """gu: (M, 2I) bf16 -> (xq (M, I), sx (M, I/128)) of silu(gate) * up."""
    _check_cuda(gu)
    if gu.dtype != torch.bfloat16 or gu.dim() != 2 or gu.stride(1) != 1:
        raise TypeError("gu must be a 2-D bf16 tensor, contiguous along its last dimension")
    M, two_i = gu.shape
    I = two_i // 2
    xq, sx = _quant_out(M, I, gu.device, True)
    lib = _lib.load()
    _lib.check(lib.fp8gq_swiglu_group_quant(_ptr(gu), gu.stride(0), M, I, _ptr(xq), _ptr(sx),
                                            _stream(gu.device)), "fp8gq_swiglu_group_quant")
    return xq, sx


def _check_gate_up(gate: torch.Tensor, up: torch.Tensor):
    _check_cuda(gate, up)
    for t, n in ((gate, "gate"), (up, "up")):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
            raise TypeError(f"{n} must be a 2-D bf16 tensor, contiguous along its last dimension")
    if gate.shape != up.shape:
        raise ShapeError(f"gate and up must have the same shape, got {tuple(gate.shape)} and {tuple(up.shape)}")
    M, I = gate.shape
    if I % GROUP:
        raise ShapeError("the SwiGLU writers need I to be a multiple of 128")
    return M, I


def fused_swiglu(gate: torch.Tensor, up: torch.Tensor, *, out=None) -> torch.Tensor:
    """gate, up: (M, I) bf16 -> bf16 silu(gate) * up, computed in fp32
    (kernels/fused_swiglu_fp8.py:48-53)."""
    M, I = _check_gate_up(gate, up)
    if out is None:
        out = torch.empty(M, I, dtype=torch.bfloat16, device=gate.device)
    lib = _lib.load()
    _lib.check(lib.fp8gq_swiglu(_ptr(gate), gate.stride(0), _ptr(up), up.stride(0), _ptr(out), out.stride(0),
                                M, I, _stream(gate.device)), "fp8gq_swiglu")
    return out


def fused_swiglu_quant(gate: torch.Tensor, up: torch.Tensor):
    """gate, up: (M, I) bf16 -> (q (M, I) float8_e4m3fn, scale (M, I/128) fp32)
    with scale = max(amax / 448, 1e-30) and q = e4m3(clamp(y / scale))
    (kernels/fused_swiglu_fp8.py:56-63)."""
    M, I = _check_gate_up(gate, up)
    q = torch.empty(M, I, dtype=torch.float8_e4m3fn, device=gate.device)
    scale = torch.empty(M, I // GROUP, dtype=torch.float32, device=gate.device)
    lib = _lib.load()
    _lib.check(lib.fp8gq_swiglu_quant(_ptr(gate), gate.stride(0), _ptr(up), up.stride(0), _ptr(q), q.stride(0),
                                      _ptr(scale), M, I, _stream(gate.device)), "fp8gq_swiglu_quant")
    return q, scale


RMS_EPS = 1e-6


def _check_norm_inputs(x, residual, weight):
    _check_cuda(x, residual, weight)
    for t, n in ((x, "x"), (residual, "residual")):
        if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
            raise TypeError(f"{n} must be a 2-D bf16 tensor, contiguous along its last dimension")
    if weight.dtype != torch.bfloat16 or weight.dim() != 1 or not weight.is_contiguous():
        raise TypeError("the norm weight must be a contiguous 1-D bf16 tensor")
    if residual.shape != x.shape or weight.shape[0] != x.shape[1]:
        raise ShapeError(f"x {tuple(x.shape)}, residual {tuple(residual.shape)} and weight "
                         f"{tuple(weight.shape)} do not match")
    M, K = x.shape
    if K % GROUP:
        raise ShapeError("K must be a multiple of 128")
    return M, K


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = RMS_EPS, *,
                out=None, residual_out=None):
    """Fused add + RMSNorm (kernels/fused_rmsnorm.py:14-27): returns
    (bf16(rmsnorm(x + residual) * weight), bf16(x + residual)); bf16 inputs,
    fp32 math in a fixed order (include/fp8gq.h, fp8gq_add_rmsnorm)."""
    M, K = _check_norm_inputs(x, residual, weight)
    if out is None:
        out = torch.empty(M, K, dtype=torch.bfloat16, device=x.device)
    if residual_out is None:
        residual_out = torch.empty(M, K, dtype=torch.bfloat16, device=x.device)
    lib = _lib.load()
    _lib.check(lib.fp8gq_add_rmsnorm(_ptr(x), x.stride(0), _ptr(residual), residual.stride(0), _ptr(weight),
                                     float(eps), _ptr(out), out.stride(0), _ptr(residual_out),
                                     residual_out.stride(0), M, K, _stream(x.device)), "fp8gq_add_rmsnorm")
    return out, residual_out


def fused_add_rmsnorm_gemv_quant(x: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor,
                                 Wq: torch.Tensor, Ws: torch.Tensor, eps: float = RMS_EPS, *, out=None,
                                 residual_out=None, return_quant: bool = False):
    """GEMV(quant(rmsnorm(x + residual) * norm_weight)) without storing the
    norm output; also returns bf16(x + residual) (the decoder's new residual).
    Returns (out, residual_out) or, with return_quant, (out, residual_out, xq, sx)."""
    M, K = _check_norm_inputs(x, residual, norm_weight)
    N = _check_weight(Wq, Ws, K)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=x.device)
    if residual_out is None:
        residual_out = torch.empty(M, K, dtype=torch.bfloat16, device=x.device)
    xq, sx = _quant_out(M, K, x.device, return_quant)
    lib = _lib.load()
    nbytes = _workspace_bytes(lib, x.device, M, N, K)
    ws_buf = workspace(x.device, nbytes) if nbytes else None
    st = lib.fp8gq_fused_add_rmsnorm_gemv_quant(
        _ptr(x), x.stride(0), _ptr(residual), residual.stride(0), _ptr(norm_weight), float(eps), _ptr(Wq),
        Wq.stride(0), _ptr(Ws), Ws.stride(0), _ptr(out), out.stride(0), _ptr(residual_out), residual_out.stride(0),
        M, N, K, _ptr(xq), _ptr(sx), _ptr(ws_buf), 0 if ws_buf is None else ws_buf.numel(), _stream(x.device))
    _lib.check(st, "fp8gq_fused_add_rmsnorm_gemv_quant")
    return (out, residual_out, xq, sx) if return_quant else (out, residual_out)


def fused_reduce_add_rmsnorm_gemv_quant(partials: torch.Tensor, residual: torch.Tensor, norm_weight: torch.Tensor,
                                        Wq: torch.Tensor, Ws: torch.Tensor, eps: float = RMS_EPS, *, out=None,
                                        residual_out=None, return_quant: bool = False, wait=None):
    """fused_add_rmsnorm_gemv_quant whose x is the sum of the partial outputs
    of a K-sharded linear: ``partials`` is [S, M, K] bf16 (S <= 8 slabs, one per
    rank, any slab stride, rows contiguous), added in slab order in fp32 before
    the residual.  ``wait`` (an fp8gq._lib.Gather of the calls that stored the
    slabs) makes the kernel wait for every rank first.  Returns (out,
    residual_out) or, with return_quant, (out, residual_out, xq, sx)."""
    if partials.dim() != 3:
        raise ShapeError("partials must be [S, M, K]")
    S = partials.shape[0]
    if not 1 <= S <= _lib.MAX_GATHER_RANKS:
        raise ShapeError(f"1 .. {_lib.MAX_GATHER_RANKS} partial slabs, got {S}")
    M, K = _check_norm_inputs(partials[0], residual, norm_weight)
    N = _check_weight(Wq, Ws, K)
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=partials.device)
    if residual_out is None:
        residual_out = torch.empty(M, K, dtype=torch.bfloat16, device=partials.device)
    xq, sx = _quant_out(M, K, partials.device, return_quant)
    lib = _lib.load()
    nbytes = _workspace_bytes(lib, partials.device, M, N, K)
    ws_buf = workspace(partials.device, nbytes) if nbytes else None
    st = lib.fp8gq_fused_reduce_add_rmsnorm_gemv_quant(
        _ptr(partials), S, partials.stride(0), partials.stride(1), _ptr(residual), residual.stride(0),
        _ptr(norm_weight), float(eps), _ptr(Wq), Wq.stride(0), _ptr(Ws), Ws.stride(0), _ptr(out), out.stride(0),
        _ptr(residual_out), residual_out.stride(0), M, N, K, _ptr(xq), _ptr(sx), wait,
        _ptr(ws_buf), 0 if ws_buf is None else ws_buf.numel(), _stream(partials.device))
    _lib.check(st, "fp8gq_fused_reduce_add_rmsnorm_gemv_quant")
    return (out, residual_out, xq, sx) if return_quant else (out, residual_out)
