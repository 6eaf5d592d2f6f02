"""The drop-in patch layer on CPU (patches/patch_fp8_fused_tail.py): routing,
fallback to the saved original, bias, output shape, install/uninstall.  The
kernel op is replaced by the oracle here; the GPU tests run the real one."""
import types

import numpy as np
import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import bf16_tensor, f32_tensor, fp8_tensor

import fp8gq.patch_fp8_fused_tail as P
from fp8gq import ops


@pytest.fixture
def fake_sglang(monkeypatch):
    """A stand-in for sglang's fp8_utils module with both originals, the fused
    op replaced by the oracle, and the CUDA check opened for CPU tensors."""
    calls = []

    def orig_cutlass(input, weight, block_size, weight_scale, input_scale, bias):
        calls.append(("cutlass", tuple(input.shape)))
        return torch.full((*input.shape[:-1], weight.shape[0]), 7.0, dtype=torch.bfloat16)

    def orig_flashinfer(input, weight, block_size, weight_scale, input_scale, bias):
        calls.append(("flashinfer", tuple(input.shape)))
        return torch.full((*input.shape[:-1], weight.shape[0]), 9.0, dtype=torch.bfloat16)

    def fake_fused(x2d, Wq, Ws):
        calls.append(("fused", tuple(x2d.shape)))
        out, _, _, _ = O.fused_gemv_quant(x2d.float().numpy(), Wq.view(torch.uint8).numpy(), Ws.numpy())
        return bf16_tensor(out)

    mod = types.ModuleType("fp8_utils")
    mod.cutlass_w8a8_block_fp8_linear_with_fallback = orig_cutlass
    mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback = orig_flashinfer
    monkeypatch.setattr(P, "_on_device", lambda *t: True)
    monkeypatch.setattr(ops, "fused_gemv_quant", fake_fused)
    yield mod, calls
    P.uninstall(mod)


def _operands(M, K=256, N=384, lead=()):
    x = bf16_tensor(O.make_activation(M, K, seed=1)).view(*lead, -1, K) if lead else \
        bf16_tensor(O.make_activation(M, K, seed=1))
    wq, ws = O.make_weight(N, K, seed=2)
    return x, fp8_tensor(wq), f32_tensor(ws)


def test_install_rebinds_and_keeps_originals(fake_sglang):
    mod, _ = fake_sglang
    orig = mod.cutlass_w8a8_block_fp8_linear_with_fallback
    assert P.install(mod) == ["cutlass_w8a8_block_fp8_linear_with_fallback",
                              "flashinfer_gemm_w8a8_block_fp8_linear_with_fallback"]
    assert mod.cutlass_w8a8_block_fp8_linear_with_fallback is P.cutlass_w8a8_block_fp8_linear_with_fallback
    assert P.install(mod)  # idempotent
    assert P._originals["cutlass_w8a8_block_fp8_linear_with_fallback"] is orig
    P.uninstall(mod)
    assert mod.cutlass_w8a8_block_fp8_linear_with_fallback is orig


def test_install_on_globals_dict(fake_sglang):
    mod, _ = fake_sglang
    g = vars(mod)
    P.install(g)
    assert g["flashinfer_gemm_w8a8_block_fp8_linear_with_fallback"] is \
        P.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback


@pytest.mark.parametrize("M, expect", [(1, "row"), (2, "tm"), (16, "tm"), (17, None), (64, None)])
def test_route_by_m(fake_sglang, M, expect):
    x, w, s = _operands(M)
    assert P.route(x, w, [128, 128], s, None) == expect


def test_route_rejects(fake_sglang):
    x, w, s = _operands(1)
    assert P.route(x, w, None, s, torch.ones(1)) is None               # static input scale
    assert P.route(x.float(), w, None, s, None) is None                # not bf16
    assert P.route(x, w.view(torch.uint8), None, s, None) is None      # not e4m3
    assert P.route(x, w, [64, 64], s, None) is None                    # other block size
    assert P.route(x, w, None, s[:1], None) is None                    # scale shape
    assert P.route(x[:, :128], w[:, :128].contiguous(), None, s[:, :1].contiguous(), None) is not None
    # layout never decides the route: an activation whose rows start 8 bytes
    # in, or whose K stride is 2, still goes to the fused path (fused_linear
    # copies it into an aligned buffer first)
    xw = torch.zeros(1, 264, dtype=torch.bfloat16)[:, 4:260]
    assert P.route(xw, w, None, s, None) == "row"
    assert P.route(torch.zeros(4, 512, dtype=torch.bfloat16)[:, ::2], w, None, s, None) == "tm"


@pytest.mark.parametrize("M, stride_k, offset", [(1, 1, 4), (3, 1, 4), (2, 2, 0), (5, 2, 1)])
def test_unaligned_routed_input_is_copied_not_sent_back(fake_sglang, M, stride_k, offset):
    mod, calls = fake_sglang
    P.install(mod)
    seen = []
    fused = ops.fused_gemv_quant

    def spy(x2d, Wq, Ws):
        seen.append((x2d.data_ptr() % 16, x2d.stride(), x2d.is_contiguous()))
        return fused(x2d, Wq, Ws)

    ops.fused_gemv_quant = spy
    try:
        x, w, s = _operands(M)
        base = torch.zeros(M * 256 * stride_k + 64, dtype=torch.bfloat16)
        xv = base[offset:offset + M * 256 * stride_k].view(M, 256 * stride_k)[:, ::stride_k]
        xv.copy_(x)
        out = mod.cutlass_w8a8_block_fp8_linear_with_fallback(xv, w, [128, 128], s, None, None)
    finally:
        ops.fused_gemv_quant = fused
    assert calls[-1][0] == "fused"
    assert seen and seen[-1][0] == 0 and seen[-1][1][1] == 1 and (seen[-1][1][0] * 2) % 16 == 0
    ref, _, _, _ = O.fused_gemv_quant(x.float().numpy(), w.view(torch.uint8).numpy(), s.numpy())
    assert torch.equal(out, bf16_tensor(ref))


def test_routed_call_uses_fused_and_adds_bias(fake_sglang):
    mod, calls = fake_sglang
    P.install(mod)
    x, w, s = _operands(1, lead=(1,))
    bias = torch.linspace(-1, 1, w.shape[0]).bfloat16()
    out = mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback(
        input=x, weight=w, block_size=[128, 128], weight_scale=s, input_scale=None, bias=bias)
    assert calls[-1] == ("fused", (1, 256))
    assert out.shape == (1, 1, 384) and out.dtype == torch.bfloat16
    ref, _, _, _ = O.fused_gemv_quant(x.view(1, 256).float().numpy(), w.view(torch.uint8).numpy(), s.numpy())
    want = (bf16_tensor(ref) + bias).view(1, 1, 384)
    assert torch.equal(out, want)


def test_unrouted_calls_go_to_the_right_original(fake_sglang):
    mod, calls = fake_sglang
    P.install(mod)
    x, w, s = _operands(32)
    out = mod.cutlass_w8a8_block_fp8_linear_with_fallback(x, w, [128, 128], s, None, None)
    assert calls[-1] == ("cutlass", (32, 256)) and float(out[0, 0]) == 7.0
    out = mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback(x, w, [128, 128], s, None, None)
    assert calls[-1] == ("flashinfer", (32, 256)) and float(out[0, 0]) == 9.0


def test_routed_errors_are_not_swallowed(fake_sglang, monkeypatch):
    mod, _ = fake_sglang
    P.install(mod)

    def boom(*a, **k):
        raise RuntimeError("kernel failed")

    monkeypatch.setattr(ops, "fused_gemv_quant", boom)
    x, w, s = _operands(1)
    with pytest.raises(RuntimeError, match="kernel failed"):
        mod.cutlass_w8a8_block_fp8_linear_with_fallback(x, w, None, s, None, None)


def test_no_original_installed_raises():
    P._originals.pop("apply_w8a8_block_fp8_linear", None)
    x = torch.zeros(32, 256, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="no original"):
        P.apply_w8a8_block_fp8_linear(x, torch.zeros(128, 256, dtype=torch.float8_e4m3fn), None,
                                      torch.ones(1, 2), None, None)
