"""Prepared launches (fp8gq_prepare_* / fp8gq_launch_plans): a call recorded
once and issued later must do exactly what the eager call does -- same
kernels, same parameters, so bit-identical outputs -- on its own, in a list,
and inside a CUDA graph."""
import ctypes

import pytest
import torch

from tests._util import assert_close, to_f32, to_u8
from oracle import fp8gq_oracle as O


def test_plan_struct_size_matches_header():
    from fp8gq import _lib
    assert ctypes.sizeof(_lib.LaunchPlan) == 4096        # FP8GQ_LAUNCH_PLAN_BYTES


def test_negative_count_is_refused_without_a_device():
    from fp8gq import _lib
    lib = _lib.load(build_if_missing=False)
    assert lib.fp8gq_launch_plans(None, -1, None) == 2   # FP8GQ_ERR_SHAPE


gpu = pytest.mark.gpu


@pytest.fixture(scope="module")
def fp8gq(cuda_device):
    import fp8gq as mod
    mod.load()
    return mod


def _weight(N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = (blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0).contiguous()
    return (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K).contiguous(), ws


def _x(M, K, seed, dev, std=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (torch.randn(M, K, generator=g, device=dev) * std).bfloat16()


# (M, K, N): row kernel, tile kernel at M = 1 (cluster split-K), small batch,
# and M = 16 (pre-quantised feed: two launches in one plan)
SHAPES = [(1, 4096, 4096), (1, 12288, 4096), (4, 2560, 4096), (16, 2560, 19456)]


@gpu
@pytest.mark.parametrize("M, K, N", SHAPES)
def test_plan_matches_eager_call(fp8gq, cuda_device, M, K, N):
    wq, ws = _weight(N, K, M + N, cuda_device)
    x = _x(M, K, K + M, cuda_device)
    eager = fp8gq.fused_gemv_quant(x, wq, ws)
    plan = fp8gq.prepare_fused_gemv_quant(x, wq, ws)
    for _ in range(2):
        plan.out.fill_(float("nan"))
        plan.run()
        torch.cuda.synchronize()
        assert torch.equal(plan.out, eager)
    _, exact, _, _ = O.fused_gemv_quant(to_f32(x), to_u8(wq), to_f32(ws))
    assert_close(to_f32(plan.out), exact, 3.0)


@gpu
@pytest.mark.parametrize("M", [1, 4])
def test_swiglu_plan_matches_eager_call(fp8gq, cuda_device, M):
    I, N = 12288, 4096
    wd, sd = _weight(N, I, 9, cuda_device)
    gu = _x(M, 2 * I, 10 + M, cuda_device, std=1.5)
    eager = fp8gq.fused_swiglu_q_gemm(gu, wd, sd)
    plan = fp8gq.prepare_fused_swiglu_q_gemm(gu, wd, sd)
    plan.run()
    torch.cuda.synchronize()
    assert torch.equal(plan.out, eager)


@gpu
def test_launch_list_of_a_chain_in_and_out_of_a_graph(fp8gq, cuda_device):
    """A decode-layer chain (qkv -> o -> gate_up -> SwiGLU down), every input
    the previous output: one LaunchList run equals the eager calls, and so does
    a CUDA graph that captured the run."""
    dev = cuda_device
    H, Q, I = 4096, 6144, 12288
    w = [_weight(Q, H, 1, dev), _weight(H, H, 2, dev), _weight(2 * I, H, 3, dev), _weight(H, I, 4, dev)]
    h = _x(1, H, 5, dev)
    qkv = torch.empty(1, Q, dtype=torch.bfloat16, device=dev)
    o = torch.empty(1, H, dtype=torch.bfloat16, device=dev)
    gu = torch.empty(1, 2 * I, dtype=torch.bfloat16, device=dev)
    d = torch.empty(1, H, dtype=torch.bfloat16, device=dev)

    def eager():
        fp8gq.fused_gemv_quant(h, *w[0], out=qkv)
        fp8gq.fused_gemv_quant(qkv[:, :H], *w[1], out=o)
        fp8gq.fused_gemv_quant(o, *w[2], out=gu)
        fp8gq.fused_swiglu_q_gemm(gu, *w[3], out=d)
        torch.cuda.synchronize()
        return [t.clone() for t in (qkv, o, gu, d)]

    ref = eager()
    plans = fp8gq.LaunchList([fp8gq.prepare_fused_gemv_quant(h, *w[0], out=qkv),
                              fp8gq.prepare_fused_gemv_quant(qkv[:, :H], *w[1], out=o),
                              fp8gq.prepare_fused_gemv_quant(o, *w[2], out=gu),
                              fp8gq.prepare_fused_swiglu_q_gemm(gu, *w[3], out=d)])
    for t in (qkv, o, gu, d):
        t.zero_()
    plans.run()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip((qkv, o, gu, d), ref))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        plans.run()
    for t in (qkv, o, gu, d):
        t.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip((qkv, o, gu, d), ref))
    del g
    assert fp8gq.device_error() == 0


@gpu
def test_invalid_plan_is_refused(fp8gq, cuda_device):
    from fp8gq import _lib
    lib = _lib.load()
    blank = (_lib.LaunchPlan * 1)()
    assert lib.fp8gq_launch_plans(blank, 1, torch.cuda.current_stream().cuda_stream) == 8   # UNSUPPORTED
    # a failed prepare leaves no launchable plan behind
    wq, ws = _weight(256, 256, 1, cuda_device)
    xbad = torch.zeros(1, 264, dtype=torch.bfloat16, device=cuda_device)[:, 4:260]
    p = _lib.LaunchPlan()
    out = torch.empty(1, 256, dtype=torch.bfloat16, device=cuda_device)
    st = lib.fp8gq_prepare_fused_gemv_quant(xbad.data_ptr(), 264, wq.data_ptr(), 256, ws.data_ptr(), 2,
                                            out.data_ptr(), 256, 1, 256, 256, None, None, None, 0, ctypes.byref(p))
    assert st == 3                                                                     # ALIGNMENT
    assert lib.fp8gq_launch_plans(ctypes.byref(p), 1, torch.cuda.current_stream().cuda_stream) == 8
