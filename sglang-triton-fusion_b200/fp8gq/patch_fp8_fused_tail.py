"""Drop-in for the reference's sglang patch ``patches/patch_fp8_fused_tail.py``.

The reference is text appended to sglang's ``fp8_utils.py``: it saves the two
block-FP8 linear entry points (``:7-8``) and rebinds their names to wrappers
(``:29-50``) that send eligible calls to the fused kernel.  sglang's
dispatch looks the names up in the module at call time, so rebinding them
before the model loads is enough.  Here the same thing is one call appended
to that file (or made on the module object)::

    from fp8gq.patch_fp8_fused_tail import install as _fp8gq_install
    _fp8gq_install(globals())

Wrappers keep the reference's signature
``(input=None, weight=None, block_size=None, weight_scale=None,
input_scale=None, bias=None, **kw) -> Tensor``.

Routing (the reference sends only M == 1 to the fused kernel,
``patches/patch_fp8_fused_tail.py:13-15``; this module also sends the small
batches the tile kernel was built for):

* routed -- ``input_scale is None``, bf16 input, e4m3 weight [N, K] with
  N, K multiples of 128, fp32 weight_scale [N/128, K/128], block_size None or
  [128, 128], CUDA tensors, M = prod(input.shape[:-1]) in [1, 16]: M == 1 ->
  row kernel (or the tile kernel for large weights), 2 <= M <= 16 -> tcgen05
  tile kernel.  The layout never decides the route: an operand the kernels
  cannot read in place (rows not 16-byte aligned, a non-unit stride along K,
  a view that does not flatten) is copied into a fresh contiguous buffer
  first, so a routed call takes the fused path whatever its strides.  A
  routed call never falls back: an error in the fused path raises (the
  reference swallows exceptions, ``:25-26``).
* everything else -- the saved original, called positionally like the
  reference does (``:37-38``, ``:49-50``).

Bias is added to the bf16 output outside the kernel (``:22-23``).
"""
from __future__ import annotations

import torch

from . import ops

MAX_FUSED_M = ops.TM

#: names of sglang's block-FP8 linear entry points that get wrapped when present
WRAPPED_NAMES = (
    "cutlass_w8a8_block_fp8_linear_with_fallback",
    "flashinfer_gemm_w8a8_block_fp8_linear_with_fallback",
    "apply_w8a8_block_fp8_linear",
)

_originals: dict = {}


def _aligned_rows(t: torch.Tensor) -> bool:
    return t.data_ptr() % 16 == 0 and (t.stride(0) * t.element_size()) % 16 == 0


def _on_device(*tensors) -> bool:
    """The fused kernels take CUDA tensors only."""
    return all(t.is_cuda for t in tensors)


def route(input, weight, block_size, weight_scale, input_scale) -> str | None:
    """'row', 'tm' or None (= call the original) for these arguments: the
    dtypes, shapes and M decide; strides and alignment do not (see
    fused_linear)."""
    if input_scale is not None or input is None or weight is None or weight_scale is None:
        return None
    if input.dtype != torch.bfloat16 or weight.dtype != torch.float8_e4m3fn:
        return None
    if weight_scale.dtype != torch.float32 or weight.dim() != 2 or weight_scale.dim() != 2:
        return None
    if not _on_device(input, weight, weight_scale):
        return None
    N, K = weight.shape
    if N % ops.GROUP or K % ops.GROUP or input.dim() < 1 or input.shape[-1] != K:
        return None
    if tuple(weight_scale.shape) != (N // ops.GROUP, K // ops.GROUP):
        return None
    if block_size is not None and [int(b) for b in block_size] != [ops.GROUP, ops.GROUP]:
        return None
    M = input.numel() // K if K else 0
    if M < 1 or M > MAX_FUSED_M:
        return None
    return "row" if M == 1 else "tm"


def _readable(t: torch.Tensor, row_align: bool = True) -> torch.Tensor:
    """t itself when the kernels can read it in place (unit stride along the
    last dimension, and 16-byte-aligned rows where row_align), else a copy into
    a fresh contiguous buffer (torch's allocator aligns it to 512 bytes)."""
    ok = t.stride(-1) == 1 and (not row_align or _aligned_rows(t))
    return t if ok else t.clone(memory_format=torch.contiguous_format)


def fused_linear(input, weight, weight_scale, bias=None) -> torch.Tensor:
    """The fused path for a routed call (patches/patch_fp8_fused_tail.py:21-24).
    Operands in a layout the kernels cannot read in place are copied first; a
    call from sglang never needs that (its activations are contiguous, its
    weights are parameters), so the copies only keep odd callers on the fused
    path instead of the original."""
    K = weight.shape[1]
    x2d = _readable(input.reshape(-1, K))
    weight = _readable(weight)
    weight_scale = _readable(weight_scale, row_align=False)
    out = ops.fused_gemv_quant(x2d, weight, weight_scale)
    if bias is not None:
        out = out + bias
    return out.view(*input.shape[:-1], weight.shape[0])


def _make_wrapper(name: str):
    def wrapper(input=None, weight=None, block_size=None, weight_scale=None,
                input_scale=None, bias=None, **kw):
        if route(input, weight, block_size, weight_scale, input_scale) is not None:
            return fused_linear(input, weight, weight_scale, bias)
        orig = _originals.get(name)
        if orig is None:
            raise RuntimeError(f"{name}: call not routed to the fused kernel and no original is "
                               f"installed (call install() on sglang's fp8_utils first)")
        return orig(input, weight, block_size, weight_scale, input_scale, bias)

    wrapper.__name__ = name
    wrapper.__qualname__ = name
    wrapper.__doc__ = f"fp8gq fused fast path in front of sglang's {name}."
    return wrapper


cutlass_w8a8_block_fp8_linear_with_fallback = _make_wrapper(WRAPPED_NAMES[0])
flashinfer_gemm_w8a8_block_fp8_linear_with_fallback = _make_wrapper(WRAPPED_NAMES[1])
apply_w8a8_block_fp8_linear = _make_wrapper(WRAPPED_NAMES[2])
_WRAPPERS = {
    WRAPPED_NAMES[0]: cutlass_w8a8_block_fp8_linear_with_fallback,
    WRAPPED_NAMES[1]: flashinfer_gemm_w8a8_block_fp8_linear_with_fallback,
    WRAPPED_NAMES[2]: apply_w8a8_block_fp8_linear,
}


def install(namespace) -> list:
    """Rebind the block-FP8 linear entry points found in ``namespace`` (a
    module or its ``globals()`` dict) to the fused wrappers, keeping the
    originals.  Idempotent.  Returns the names that were wrapped."""
    ns = namespace if isinstance(namespace, dict) else vars(namespace)
    done = []
    for name in WRAPPED_NAMES:
        cur = ns.get(name)
        if cur is None:
            continue
        if cur is not _WRAPPERS[name]:
            _originals[name] = cur
            ns[name] = _WRAPPERS[name]
        done.append(name)
    return done


def uninstall(namespace) -> None:
    """Put the saved originals back into ``namespace``."""
    ns = namespace if isinstance(namespace, dict) else vars(namespace)
    for name, orig in list(_originals.items()):
        if ns.get(name) is _WRAPPERS[name]:
            ns[name] = orig
        _originals.pop(name, None)
