"""Opt-in MLP hook: gate_up -> SwiGLU + quant + down_proj in one kernel.

The reference tried this as a patch of sglang's ``Qwen2MLP.forward`` (which
Qwen3 reuses): at M == 1, gate_up through the patched block-FP8 linear, then
``fused_swiglu_q_gemm`` -- silu(gate) * up, the 128-group FP8 quant and the
down_proj GEMV in one kernel -- instead of ``act_fn`` followed by
``down_proj`` (docs/TRITON_KERNELS.md, section 15; the reference reverted it
after measuring no end-to-end gain on its GPU).  Here it is an explicit,
reversible hook on the MLP class::

    from sglang.srt.models.qwen2 import Qwen2MLP
    from fp8gq.patch_mlp import install_mlp_hook
    install_mlp_hook(Qwen2MLP)

The hooked ``forward(x)`` takes the fused path only when the call is the plain
MLP the kernel replaces: no extra arguments; ``act_fn`` is a SiLU-and-mul
(``[gate | up]`` layout); ``down_proj`` holds a block-FP8 weight (e4m3 [N, I]
with fp32 ``weight_scale_inv`` [N/128, I/128], dynamic activation scale);
M = tokens in 1..16; bf16 CUDA tensors; and, if ``down_proj`` reduces its
output over tensor-parallel ranks, an ``all_reduce`` callable was given to
``install_mlp_hook``.  Anything else runs the original forward.  A call that
takes the fused path never falls back: errors raise.
"""
from __future__ import annotations

import torch

from . import ops

MAX_FUSED_M = ops.TM

_originals: dict = {}


def _on_device(*tensors) -> bool:
    """The fused kernels take CUDA tensors only."""
    return all(t.is_cuda for t in tensors)


def _is_silu_and_mul(act) -> bool:
    return type(act).__name__ in ("SiluAndMul", "SiLUAndMul")


def route(mlp, x, args=(), kwargs=None) -> bool:
    """Whether the hooked forward takes the fused gate_up -> SwiGLU+quant+down path."""
    if args or kwargs:
        return False
    down = getattr(mlp, "down_proj", None)
    if down is None or not hasattr(mlp, "gate_up_proj") or not _is_silu_and_mul(getattr(mlp, "act_fn", None)):
        return False
    w = getattr(down, "weight", None)
    s = getattr(down, "weight_scale_inv", None)
    if not isinstance(w, torch.Tensor) or not isinstance(s, torch.Tensor):
        return False
    if w.dtype != torch.float8_e4m3fn or s.dtype != torch.float32 or w.dim() != 2 or s.dim() != 2:
        return False
    if getattr(down, "input_scale", None) is not None:
        return False
    N, I = w.shape
    if N % ops.GROUP or I % ops.GROUP or tuple(s.shape) != (N // ops.GROUP, I // ops.GROUP):
        return False
    if not isinstance(x, torch.Tensor) or x.dtype != torch.bfloat16 or not _on_device(x, w, s):
        return False
    M = x.numel() // x.shape[-1] if x.dim() >= 1 and x.shape[-1] else 0
    if not 1 <= M <= MAX_FUSED_M:
        return False
    needs_reduce = bool(getattr(down, "reduce_results", False)) and int(getattr(down, "tp_size", 1)) > 1
    if needs_reduce and _originals.get(type(mlp), {}).get("all_reduce") is None:
        return False
    return True


def _fused_forward(mlp, x):
    down = mlp.down_proj
    gate_up = mlp.gate_up_proj(x)
    if isinstance(gate_up, tuple):            # sglang linears return (output, bias)
        gate_up = gate_up[0]
    two_i = gate_up.shape[-1]
    gu = gate_up.reshape(-1, two_i)
    if gu.stride(-1) != 1 or gu.data_ptr() % 16 or (gu.stride(0) * 2) % 16:
        gu = gu.clone(memory_format=torch.contiguous_format)
    w = down.weight
    if w.stride(1) != 1 or w.data_ptr() % 16 or w.stride(0) % 16:
        w = w.contiguous()
    out = ops.fused_swiglu_q_gemm(gu, w, down.weight_scale_inv.contiguous())
    bias = getattr(down, "bias", None)
    if bias is not None and not getattr(down, "skip_bias_add", False):
        out = out + bias
    if bool(getattr(down, "reduce_results", False)) and int(getattr(down, "tp_size", 1)) > 1:
        out = _originals[type(mlp)]["all_reduce"](out)
    return out.view(*x.shape[:-1], w.shape[0])


def install_mlp_hook(mlp_cls, all_reduce=None) -> None:
    """Wrap ``mlp_cls.forward`` (idempotent).  ``all_reduce`` (out -> out) is
    applied after down_proj when down_proj reduces over tensor-parallel ranks;
    without it such calls run the original forward."""
    if mlp_cls in _originals:
        _originals[mlp_cls]["all_reduce"] = all_reduce
        return
    orig = mlp_cls.forward

    def forward(self, x, *args, **kwargs):
        if route(self, x, args, kwargs):
            return _fused_forward(self, x)
        return orig(self, x, *args, **kwargs)

    forward.__name__ = getattr(orig, "__name__", "forward")
    forward.__doc__ = "fp8gq: gate_up, then SwiGLU + quant + down_proj in one kernel for M <= 16."
    _originals[mlp_cls] = {"forward": orig, "all_reduce": all_reduce}
    mlp_cls.forward = forward


def uninstall_mlp_hook(mlp_cls) -> None:
    """Put the original forward back."""
    ent = _originals.pop(mlp_cls, None)
    if ent is not None:
        mlp_cls.forward = ent["forward"]
