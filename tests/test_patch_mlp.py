"""The opt-in MLP hook (fp8gq.patch_mlp): gate_up, then SwiGLU + quant +
down_proj in one kernel, in place of act_fn followed by down_proj (the
reference's reverted Qwen2MLP.forward patch, docs/TRITON_KERNELS.md section
15).  On CPU the kernel is replaced by the oracle; the GPU test runs it."""
import numpy as np
import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import bf16_tensor, f32_tensor, fp8_tensor, to_f32, to_u8

import fp8gq.patch_mlp as PM
from fp8gq import ops


class SiluAndMul(torch.nn.Module):
    def forward(self, gu):
        i = gu.shape[-1] // 2
        g, u = gu[..., :i].float(), gu[..., i:].float()
        return (g * torch.sigmoid(g) * u).bfloat16()


class FP8Linear(torch.nn.Module):
    """Stand-in for sglang's block-FP8 linear: returns (out, None) and holds
    weight / weight_scale_inv like sglang's Fp8LinearMethod layers."""

    def __init__(self, wq, ws, reduce_results=False, tp_size=1):
        super().__init__()
        self.weight, self.weight_scale_inv = wq, ws
        self.input_scale = None
        self.bias = None
        self.reduce_results, self.tp_size = reduce_results, tp_size
        self.calls = 0

    def forward(self, x):
        self.calls += 1
        x2 = x.reshape(-1, x.shape[-1])
        if x2.is_cuda:
            out = ops.fused_gemv_quant(x2.contiguous(), self.weight, self.weight_scale_inv)
        else:
            out = bf16_tensor(O.fused_gemv_quant(x2.float().numpy(), to_u8(self.weight), to_f32(self.weight_scale_inv))[0])
        return out.view(*x.shape[:-1], -1), None


class StubMLP(torch.nn.Module):
    def __init__(self, wgu, sgu, wd, sd, **down_kw):
        super().__init__()
        self.gate_up_proj = FP8Linear(wgu, sgu)
        self.down_proj = FP8Linear(wd, sd, **down_kw)
        self.act_fn = SiluAndMul()

    def forward(self, x, *extra):
        gu, _ = self.gate_up_proj(x)
        out, _ = self.down_proj(self.act_fn(gu))
        return out


def _weights(H, I, dev="cpu"):
    wgu, sgu = O.make_weight(2 * I, H, seed=3)
    wd, sd = O.make_weight(H, I, seed=4)
    return fp8_tensor(wgu, dev), f32_tensor(sgu, dev), fp8_tensor(wd, dev), f32_tensor(sd, dev)


@pytest.fixture
def cpu_kernel(monkeypatch):
    """The CUDA check opened for CPU tensors and the fused kernel replaced by
    the oracle, recording its calls."""
    calls = []

    def fake(gu, wd, sd):
        calls.append(tuple(gu.shape))
        return bf16_tensor(O.fused_swiglu_q_gemm(gu.float().numpy(), to_u8(wd), to_f32(sd))[0])

    monkeypatch.setattr(PM, "_on_device", lambda *t: True)
    monkeypatch.setattr(ops, "fused_swiglu_q_gemm", fake)
    yield calls
    PM.uninstall_mlp_hook(StubMLP)


@pytest.mark.parametrize("M", [1, 3, 16])
def test_hook_routes_small_m_through_the_fused_kernel(cpu_kernel, M):
    H, I = 256, 384
    mlp = StubMLP(*_weights(H, I))
    x = bf16_tensor(O.make_activation(M, H, seed=5)).view(M, 1, H)
    PM.install_mlp_hook(StubMLP)
    out = mlp(x)
    assert cpu_kernel == [(M, 2 * I)] and mlp.down_proj.calls == 0 and mlp.gate_up_proj.calls == 1
    assert out.shape == (M, 1, H)
    gu, _ = mlp.gate_up_proj(x)
    ref = O.fused_swiglu_q_gemm(gu.view(M, 2 * I).float().numpy(), to_u8(mlp.down_proj.weight),
                                to_f32(mlp.down_proj.weight_scale_inv))[0]
    assert np.array_equal(to_f32(out).reshape(M, H), ref)


def test_hook_leaves_other_calls_to_the_original(cpu_kernel):
    H, I = 256, 384
    mlp = StubMLP(*_weights(H, I))
    PM.install_mlp_hook(StubMLP)
    big = bf16_tensor(O.make_activation(17, H, seed=6))
    mlp(big)                                                    # M > 16
    mlp(bf16_tensor(O.make_activation(1, H, seed=7)), "extra")  # an extra argument
    assert cpu_kernel == [] and mlp.down_proj.calls == 2
    tp = StubMLP(*_weights(H, I), reduce_results=True, tp_size=2)
    tp(bf16_tensor(O.make_activation(1, H, seed=8)))            # TP reduce without an all_reduce
    assert cpu_kernel == [] and tp.down_proj.calls == 1
    PM.install_mlp_hook(StubMLP, all_reduce=lambda t: t * 2)    # with one: fused, then reduced
    out = tp(bf16_tensor(O.make_activation(1, H, seed=8)))
    assert cpu_kernel == [(1, 2 * I)] and tp.down_proj.calls == 1
    assert torch.isfinite(out.float()).all()


def test_uninstall_restores_forward(cpu_kernel):
    orig = StubMLP.forward
    PM.install_mlp_hook(StubMLP)
    assert StubMLP.forward is not orig
    PM.install_mlp_hook(StubMLP)                                # idempotent
    PM.uninstall_mlp_hook(StubMLP)
    assert StubMLP.forward is orig


@pytest.mark.gpu
def test_hook_on_gpu_matches_oracle(cuda_device):
    import fp8gq
    fp8gq.load()
    H, I = 4096, 12288
    mlp = StubMLP(*_weights(H, I, cuda_device))
    PM.install_mlp_hook(StubMLP)
    try:
        for M in (1, 4):
            x = bf16_tensor(O.make_activation(M, H, seed=9 + M), cuda_device)
            out = mlp(x)
            gu, _ = mlp.gate_up_proj(x)
            _, exact, _, _ = O.fused_swiglu_q_gemm(to_f32(gu), to_u8(mlp.down_proj.weight),
                                                    to_f32(mlp.down_proj.weight_scale_inv))
            assert mlp.down_proj.calls == 0
            assert torch.equal(out, fp8gq.fused_swiglu_q_gemm(gu, mlp.down_proj.weight,
                                                               mlp.down_proj.weight_scale_inv))
            got = to_f32(out).astype(np.float64)
            assert O.rms_tolerance_ok(got, exact)
            assert np.all(np.abs(got - exact) <= O.ref_atol(exact, 3.0))
    finally:
        PM.uninstall_mlp_hook(StubMLP)
