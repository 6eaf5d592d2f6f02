"""Parity of the CUDA kernels (through the C ABI, via fp8gq.ops) against the
CPU oracle: quantised activation bytes and scales bit-exact, outputs within
a relative tolerance (rtol 1e-2, atol 1e-2 * RMS) and within the
reference self-tests' ulp tolerance (2 bf16 ulp + 1e-3 for the row and
SwiGLU kernels, kernels/fused_gemv_quant.py:107-108; 3 ulp + 1e-3 for the
tile kernel, kernels/fused_gemv_quant_tm.py:138-140)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import (assert_close, bf16_bits_tensor, bf16_tensor, f32_tensor, fp8_tensor, to_f32,
                         to_u8)

pytestmark = pytest.mark.gpu

GOLDEN = sorted(p for p in (Path(__file__).parent / "golden").glob("*.npz") if not p.stem.startswith("writer_"))
WRITER_GOLDEN = sorted((Path(__file__).parent / "golden").glob("writer_*.npz"))

# the Qwen3-8B decode linears (K, N) and the Qwen3-4B small-batch shapes
QWEN3_8B = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 24576), "down": (12288, 4096)}
QWEN3_4B = {"q": (2560, 4096), "gate_up": (2560, 19456), "down": (9728, 2560)}


@pytest.fixture(scope="module")
def fp8gq(cuda_device):
    import fp8gq as mod
    mod.load()
    return mod


def gpu_weight(N, K, seed, dev):
    """Seeded e4m3 weight [N, K] with 128x128 block scales, made on the GPU
    (N(0, 0.02^2) in bf16, ws = amax/448, RNE cast)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0
    q = (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K)
    return q.contiguous(), ws.contiguous()


def gpu_activation(M, K, seed, dev, std=1.0, outliers=True):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev) * std
    if outliers:
        ch = torch.randperm(K, generator=g, device=dev)[: max(1, round(0.01 * K))]
        x[:, ch] *= 20.0
    return x.bfloat16().contiguous()


def oracle_of(x, wq, ws, swiglu=False):
    fn = O.fused_swiglu_q_gemm if swiglu else O.fused_gemv_quant
    return fn(to_f32(x), to_u8(wq), to_f32(ws))


# ---------------------------------------------------------------- quant --

@pytest.mark.parametrize("M, K", [(1, 4096), (16, 2560), (3, 12288), (5, 128)])
def test_group_quant_bit_exact(fp8gq, cuda_device, M, K):
    x = gpu_activation(M, K, 100 + M, cuda_device)
    xq, sx = fp8gq.group_quant(x)
    rq, rs = O.group_quant(to_f32(x))
    assert np.array_equal(to_u8(xq), rq)
    assert np.array_equal(to_f32(sx), rs)


def test_group_quant_special_values(fp8gq, cuda_device):
    x = np.zeros((2, 640), np.float32)
    x[0, 128:256] = 3.0
    x[0, 130] = -400.0                                     # saturates to -448
    x[0, 256:384] = np.linspace(-1e-3, 1e-3, 128)           # subnormal codes and signed zeros
    x[0, 300] = 1.0
    x[0, 384:512] = 1e30                                     # huge but finite in bf16
    x[1, :] = np.float32(2.0) ** -120                        # tiny: below the eps floor
    x[1, 512:640] = -0.0
    x = O.bf16_round(x)
    xt = bf16_tensor(x, cuda_device)
    xq, sx = fp8gq.group_quant(xt)
    rq, rs = O.group_quant(x)
    assert np.array_equal(to_u8(xq), rq)
    assert np.array_equal(to_f32(sx), rs)
    assert to_u8(xq)[0, 130] == 0xFE


@pytest.mark.parametrize("M, I", [(1, 12288), (4, 2560)])
def test_swiglu_group_quant_bit_exact(fp8gq, cuda_device, M, I):
    gu = gpu_activation(M, 2 * I, 7, cuda_device, std=1.5, outliers=False)
    gu[:, :64] = -50.0           # silu -> ~0, stays finite
    gu[:, 64:128] = 20.0
    gu[:, I + 64:I + 128] = 20.0  # silu(20) * 20 = 400 -> group max at 448
    xq, sx = fp8gq.swiglu_group_quant(gu)
    rq, rs, _ = O.swiglu_quant(to_f32(gu))
    assert np.array_equal(to_u8(xq), rq)
    assert np.array_equal(to_f32(sx), rs)


# ------------------------------------------------------- golden fixtures --

@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_fixtures(fp8gq, cuda_device, path):
    """Every golden case through the routed entry point (M == 1 -> row
    kernel, M > 1 -> tile kernel), against the reference kernels' own output."""
    d = np.load(path)
    x = bf16_bits_tensor(d["x_bf16"], cuda_device)
    wq = fp8_tensor(d["wq"], cuda_device)
    ws = f32_tensor(d["ws"], cuda_device)
    swiglu = str(d["kind"]) == "swiglu"
    fn = fp8gq.fused_swiglu_q_gemm if swiglu else fp8gq.fused_gemv_quant
    out, xq, sx = fn(x, wq, ws, return_quant=True)
    ref_out, exact, rq, rs = oracle_of(x, wq, ws, swiglu)
    assert np.array_equal(to_u8(xq), rq), "quantised bytes differ from the oracle"
    assert np.array_equal(to_f32(sx), rs), "scales differ from the oracle"
    golden = O.bf16_from_bits(d["out_bf16"])
    ulps = 2.0 if x.shape[0] == 1 else 3.0
    assert_close(to_f32(out), exact, ulps)
    assert np.max(np.abs(to_f32(out) - golden)) <= O.ref_atol(golden, ulps)


# ------------------------------------------------------------ row kernel --

@pytest.mark.parametrize("name", list(QWEN3_8B))
def test_row_kernel_qwen3_8b(fp8gq, cuda_device, name):
    K, N = QWEN3_8B[name]
    x = gpu_activation(1, K, 1, cuda_device)
    wq, ws = gpu_weight(N, K, 2, cuda_device)
    out, xq, sx = fp8gq.fused_gemv_quant(x, wq, ws, return_quant=True, kernel="row")
    _, exact, rq, rs = oracle_of(x, wq, ws)
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    assert_close(to_f32(out), exact, 2.0)


@pytest.mark.parametrize("K, N", [(128, 128), (256, 384), (2560, 4096), (9728, 2560), (1152, 1280),
                                  (16384, 512), (49152, 256)])
def test_row_kernel_shapes(fp8gq, cuda_device, K, N):
    x = gpu_activation(1, K, K + N, cuda_device)
    wq, ws = gpu_weight(N, K, 3, cuda_device)
    out = fp8gq.fused_gemv_quant(x, wq, ws, kernel="row")
    _, exact, _, _ = oracle_of(x, wq, ws)
    assert_close(to_f32(out), exact, 2.0)


def test_row_kernel_strided_weight(fp8gq, cuda_device):
    """Weight rows padded (ldw > K): the per-row bulk-copy path."""
    K, N = 1024, 768
    x = gpu_activation(1, K, 5, cuda_device)
    wq, ws = gpu_weight(N, K, 6, cuda_device)
    big = torch.zeros(N, K + 256, dtype=torch.float8_e4m3fn, device=cuda_device)
    big[:, :K] = wq
    out = fp8gq.fused_gemv_quant(x, big[:, :K], ws)
    _, exact, _, _ = oracle_of(x, wq, ws)
    assert_close(to_f32(out), exact, 2.0)


def test_row_kernel_deterministic(fp8gq, cuda_device):
    x = gpu_activation(1, 4096, 9, cuda_device)
    wq, ws = gpu_weight(6144, 4096, 10, cuda_device)
    a = fp8gq.fused_gemv_quant(x, wq, ws)
    b = fp8gq.fused_gemv_quant(x, wq, ws)
    assert torch.equal(a, b)


# ----------------------------------------------------------- tile kernel --

@pytest.mark.parametrize("M", [2, 4, 8, 16])
@pytest.mark.parametrize("name", list(QWEN3_4B))
def test_tile_kernel_qwen3_4b(fp8gq, cuda_device, M, name):
    K, N = QWEN3_4B[name]
    x = gpu_activation(M, K, 20 + M, cuda_device)
    wq, ws = gpu_weight(N, K, 21, cuda_device)
    out, xq, sx = fp8gq.fused_gemv_quant(x, wq, ws, return_quant=True)
    _, exact, rq, rs = oracle_of(x, wq, ws)
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    assert_close(to_f32(out), exact, 3.0)


@pytest.mark.parametrize("M", [1, 17, 33, 64, 65, 100])
def test_tile_kernel_token_tiles(fp8gq, cuda_device, M):
    K, N = 1024, 1280
    x = gpu_activation(M, K, 30 + M, cuda_device)
    wq, ws = gpu_weight(N, K, 31, cuda_device)
    out = fp8gq.fused_gemv_quant(x, wq, ws, kernel="tm")
    _, exact, _, _ = oracle_of(x, wq, ws)
    assert_close(to_f32(out), exact, 3.0)


@pytest.mark.parametrize("name", list(QWEN3_8B))
def test_tile_kernel_m1_matches_row_kernel(fp8gq, cuda_device, name):
    K, N = QWEN3_8B[name]
    x = gpu_activation(1, K, 40, cuda_device)
    wq, ws = gpu_weight(N, K, 41, cuda_device)
    tm = fp8gq.fused_gemv_quant(x, wq, ws, kernel="tm")
    _, exact, _, _ = oracle_of(x, wq, ws)
    assert_close(to_f32(tm), exact, 3.0)


def test_tile_kernel_strides_and_determinism(fp8gq, cuda_device):
    M, K, N = 6, 2048, 1536
    xb = gpu_activation(M, K + 64, 50, cuda_device)
    x = xb[:, :K]                                         # ldx = K + 64
    wq, ws = gpu_weight(N, K, 51, cuda_device)
    out_big = torch.full((M, N + 128), 3.0, dtype=torch.bfloat16, device=cuda_device)
    fp8gq.fused_gemv_quant(x, wq, ws, out=out_big[:, :N])
    a = out_big[:, :N].clone()
    fp8gq.fused_gemv_quant(x, wq, ws, out=out_big[:, :N])
    assert torch.equal(a, out_big[:, :N])                 # split-K fixup is deterministic
    assert torch.all(out_big[:, N:] == 3.0)               # nothing written past ldo's row
    _, exact, _, _ = oracle_of(x.contiguous(), wq, ws)
    assert_close(to_f32(a), exact, 3.0)


@pytest.mark.parametrize("M, K, N, swiglu", [
    (1, 4096, 24576, False),    # one CTA per row block, whole K range resident (slot = K block)
    (1, 4096, 4096, False),     # K range split 8 ways: a cluster of 8 CTAs per row block (slot = tile)
    (2, 4096, 6144, False),     # a cluster of 4
    (3, 2560, 4096, False),     # 20 K blocks over clusters of 8: uneven K ranges (2 or 3 K blocks)
    (4, 4096, 1152, False),     # 9 row blocks: a cluster of 8 per row block, one CTA per SM
    (1, 12288, 512, False),     # 4 row blocks x 96 K blocks: a cluster of 16 (non-portable) per row block
    (3, 12288, 1024, False),    # 8 row blocks: clusters of 16 where they all fit, else of 8
    (4, 4096, 512, True),       # SwiGLU with a cluster of 16
    (2, 10368, 896, False),     # 7 row blocks x 81 K blocks: clusters of 16 with uneven K ranges
    (16, 1024, 1280, False),    # 16 tokens x 8 K blocks: a large resident footprint
    (16, 4096, 6144, False),    # 16 tokens x 8 K blocks per CTA: the resident feed fits
    (16, 4096, 24576, False),   # 16 tokens x 32 K blocks: only the pre-quantised feed fits
    (12, 12288, 4096, True),    # pre-quantised SwiGLU feed
    (40, 2048, 2560, False),    # 64-token tile
    (6, 3072, 4096, False),     # groups of 2 K blocks, 2 idle token rows each
    (8, 4096, 24576, False),
    (1, 12288, 4096, True),
    (2, 12288, 4096, True),
    (3, 2560, 2560, True),
])
def test_tile_kernel_strategies_agree(fp8gq, cuda_device, M, K, N, swiglu):
    """The activation feed (resident / streaming / pre-quantised) and the
    split-K reduction (cluster / workspace) change where data waits, not what
    is computed: the same MMAs on the same bytes, partial sums added in the
    same order.  All combinations agree bit for bit, with each other and
    (quant outputs) with the oracle.  The pre-quantised feed places each
    token of an accumulator group by loading its B tile from a negative row
    of the activation tensor; M = 1 .. 8 cover groups of 16 down to 2 K
    blocks, non-power-of-two M included."""
    xb = gpu_activation(M, (2 * K if swiglu else K) + 64, 130 + M, cuda_device, std=1.5 if swiglu else 1.0,
                        outliers=not swiglu)
    x = xb[:, :2 * K] if swiglu else xb[:, :K]               # a row stride longer than the row
    wq, ws = gpu_weight(N, K, 131, cuda_device)
    run = fp8gq.fused_swiglu_q_gemm if swiglu else (lambda *a, **k: fp8gq.fused_gemv_quant(*a, kernel="tm", **k))
    res = {}
    for flags in (0, fp8gq.TM_STREAM_ACTIVATIONS, fp8gq.TM_WORKSPACE_SPLITK,
                  fp8gq.TM_STREAM_ACTIVATIONS | fp8gq.TM_WORKSPACE_SPLITK,
                  fp8gq.TM_PREQUANT_ACTIVATIONS, fp8gq.TM_PREQUANT_ACTIVATIONS | fp8gq.TM_WORKSPACE_SPLITK,
                  fp8gq.TM_RESIDENT_ACTIVATIONS):
        prev = fp8gq.set_tm_options(flags)
        try:
            res[flags] = [t.clone() for t in run(x, wq, ws, return_quant=True)]
        finally:
            fp8gq.set_tm_options(prev)
    for flags in list(res)[1:]:
        for a, b in zip(res[0], res[flags]):
            assert torch.equal(a, b), flags
    _, exact, rq, rs = oracle_of(x.contiguous(), wq, ws, swiglu=swiglu)
    out, xq, sx = res[0]
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    assert_close(to_f32(out), exact, 3.0)


def test_tile_options_reject_unknown_bits(fp8gq, cuda_device):
    for flags in (16, fp8gq.TM_STREAM_ACTIVATIONS | fp8gq.TM_PREQUANT_ACTIVATIONS,
                  fp8gq.TM_PREQUANT_ACTIVATIONS | fp8gq.TM_RESIDENT_ACTIVATIONS):
        with pytest.raises(ValueError):
            fp8gq.set_tm_options(flags)
    assert fp8gq.set_tm_options(0) == 0


def test_tile_kernel_workspace_shared_across_shapes(fp8gq, cuda_device):
    """Small-N and large-N calls alternate on one workspace: the split-K
    counters of one shape must not be overwritten by another's partial sums."""
    cases = [(2, 1024, 1280), (4, 4096, 24576), (3, 2560, 4096), (1, 4096, 24576), (16, 1024, 512)]
    ops = []
    for i, (M, K, N) in enumerate(cases):
        x = gpu_activation(M, K, 90 + i, cuda_device)
        wq, ws = gpu_weight(N, K, 95 + i, cuda_device)
        ops.append((x, wq, ws, oracle_of(x, wq, ws)[1]))
    for _ in range(2):
        for x, wq, ws, exact in ops:
            out = fp8gq.fused_gemv_quant(x, wq, ws, kernel="tm")
            assert_close(to_f32(out), exact, 3.0)


# ---------------------------------------------------------------- SwiGLU --

@pytest.mark.parametrize("M", [1, 2, 16])
def test_swiglu_down_proj(fp8gq, cuda_device, M):
    I, N = 12288, 4096
    gu = gpu_activation(M, 2 * I, 60 + M, cuda_device, std=1.5, outliers=False)
    wq, ws = gpu_weight(N, I, 61, cuda_device)
    out, xq, sx = fp8gq.fused_swiglu_q_gemm(gu, wq, ws, return_quant=True)
    _, exact, rq, rs = oracle_of(gu, wq, ws, swiglu=True)
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    # 12288 -> 4096 is routed to the tile kernel at every M (its tolerance)
    assert_close(to_f32(out), exact, 3.0)


# ------------------------------------------------------------- lm_head --

@pytest.mark.parametrize("M", [1, 4])
def test_lm_head_vocab_rows(fp8gq, cuda_device, M):
    """lm_head-shaped GEMV: N = 151936 vocabulary rows (1187 row blocks, a
    stream-K grid with CTA ranges crossing row blocks); K cut to 1024 so the
    float64 oracle stays quick.  kernels/fused_gemv_quant.py:82 and
    kernels/fused_gemv_quant_tm.py:123 bench this shape."""
    K, N = 1024, 151936
    x = gpu_activation(M, K, 400 + M, cuda_device)
    wq, ws = gpu_weight(N, K, 401, cuda_device)
    out, xq, sx = fp8gq.fused_gemv_quant(x, wq, ws, return_quant=True)
    _, exact, rq, rs = oracle_of(x, wq, ws)
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    assert_close(to_f32(out), exact, 3.0)


# ---------------------------------------------------- add + RMSNorm --

def _norm_inputs(M, K, seed, dev, scale=1.0):
    x = gpu_activation(M, K, seed, dev, std=scale, outliers=False)
    r = gpu_activation(M, K, seed + 1, dev, std=scale, outliers=False)
    g = torch.Generator(device=dev).manual_seed(seed + 2)
    w = (torch.randn(K, generator=g, device=dev) * 0.1 + 1.0).bfloat16()
    return x, r, w


@pytest.mark.parametrize("M, K", [(1, 4096), (4, 2560), (16, 12288), (3, 128)])
def test_add_rmsnorm_bit_exact(fp8gq, cuda_device, M, K):
    x, r, w = _norm_inputs(M, K, 500 + M, cuda_device)
    h, res = fp8gq.add_rmsnorm(x, r, w)
    rh, rres, _ = O.add_rmsnorm(to_f32(x), to_f32(r), to_f32(w))
    assert np.array_equal(to_f32(h), rh)
    assert np.array_equal(to_f32(res), rres)


@pytest.mark.parametrize("M, K, N", [
    (1, 4096, 6144),    # tile kernel, resident
    (1, 4096, 4096),    # row kernel
    (1, 2560, 4096),    # row kernel, Qwen3-4B hidden
    (4, 4096, 24576),   # tile kernel at M = 4
    (16, 4096, 6144),   # M = 16: the norm forces one CTA per SM so the activation stays resident
    (8, 2560, 19456),
])
def test_fused_add_rmsnorm_gemv(fp8gq, cuda_device, M, K, N):
    """The prologue computes the same norm bits as the stand-alone kernel, so
    the quantised bytes equal those of the unfused chain and of the oracle."""
    x, r, w = _norm_inputs(M, K, 600 + M + K, cuda_device)
    wq, ws = gpu_weight(N, K, 601, cuda_device)
    out, res, xq, sx = fp8gq.fused_add_rmsnorm_gemv_quant(x, r, w, wq, ws, return_quant=True)
    h, res2 = fp8gq.add_rmsnorm(x, r, w)
    out2, xq2, sx2 = fp8gq.fused_gemv_quant(h, wq, ws, return_quant=True)
    assert torch.equal(xq, xq2) and torch.equal(sx, sx2)
    assert torch.equal(res, res2)
    _, exact, rq, rs, rres = O.fused_add_rmsnorm_gemv_quant(to_f32(x), to_f32(r), to_f32(w), to_u8(wq), to_f32(ws))
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    assert np.array_equal(to_f32(res), rres)
    assert_close(to_f32(out), exact, 3.0)
    assert_close(to_f32(out2), exact, 3.0)


def test_add_rmsnorm_stress_battery(fp8gq, cuda_device):
    """benchmarks/stress_tests.py:122-146 on the GPU norm and the fused path."""
    K = 2560
    z = torch.zeros(4, K, dtype=torch.bfloat16, device=cuda_device)
    w = (torch.randn(K, device=cuda_device) * 0.1).bfloat16()
    h, res = fp8gq.add_rmsnorm(z, z, w)
    assert bool((h == 0).all()) and bool((res == 0).all())
    x, r, _ = _norm_inputs(8, K, 700, cuda_device, scale=1e6)
    h, res = fp8gq.add_rmsnorm(x, r, w)
    ref = torch.nn.functional.rms_norm(x.float() + r.float(), (K,), w.float(), 1e-6)
    assert bool(torch.isfinite(h).all())
    assert torch.allclose(h.float(), ref, rtol=1e-2, atol=1e-2)
    ones = torch.ones(K, dtype=torch.bfloat16, device=cuda_device)
    x, r, _ = _norm_inputs(4, K, 710, cuda_device)
    h, _ = fp8gq.add_rmsnorm(x, r, ones)
    s = x.float() + r.float()
    manual = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6)
    assert torch.allclose(h.float(), manual, rtol=1e-2, atol=1e-2)
    wq, ws = gpu_weight(2560, K, 711, cuda_device)
    with pytest.raises(fp8gq.Fp8gqError):                 # residual_out may not alias residual
        fp8gq.fused_add_rmsnorm_gemv_quant(x, r, ones, wq, ws, residual_out=r)


# ------------------- reduce + add + RMSNorm prologue (paired tensor parallel) --

@pytest.mark.parametrize("M, K, N, S, gap", [
    (1, 4096, 6144, 3, 0),      # tile kernel, three partial slabs back to back
    (1, 4096, 4096, 8, 256),    # row kernel, eight slabs with a gap between them
    (1, 4096, 3072, 2, 0),      # row kernel: the gate_up slice of a rank at 8-way tensor parallel
    (4, 4096, 24576, 5, 128),   # tile kernel, M = 4
    (16, 2560, 4096, 8, 0),
])
def test_fused_reduce_add_rmsnorm_gemv(fp8gq, cuda_device, M, K, N, S, gap):
    """x = the sum of S partial slabs in slab order, then + residual: residual
    output and quantised bytes bit-exact against the oracle, output within
    the GEMV tolerance."""
    store = torch.zeros(S, M * K + gap, dtype=torch.bfloat16, device=cuda_device)
    parts = store[:, :M * K].view(S, M, K)
    for i in range(S):
        parts[i].copy_(gpu_activation(M, K, 800 + 10 * i + M, cuda_device, std=0.5))
    _, r, w = _norm_inputs(M, K, 850 + M, cuda_device)
    wq, ws = gpu_weight(N, K, 851, cuda_device)
    out, res, xq, sx = fp8gq.fused_reduce_add_rmsnorm_gemv_quant(parts, r, w, wq, ws, return_quant=True)
    _, exact, rq, rs, rres = O.fused_reduce_add_rmsnorm_gemv_quant([to_f32(parts[i]) for i in range(S)], to_f32(r),
                                                                   to_f32(w), to_u8(wq), to_f32(ws))
    assert np.array_equal(to_f32(res), rres)
    assert np.array_equal(to_u8(xq), rq) and np.array_equal(to_f32(sx), rs)
    assert_close(to_f32(out), exact, 3.0)


def test_fused_reduce_one_slab_is_add_rmsnorm(fp8gq, cuda_device):
    """One slab is the plain fused add + RMSNorm, bit for bit."""
    x, r, w = _norm_inputs(1, 4096, 860, cuda_device)
    wq, ws = gpu_weight(6144, 4096, 861, cuda_device)
    a = fp8gq.fused_add_rmsnorm_gemv_quant(x, r, w, wq, ws, return_quant=True)
    b = fp8gq.fused_reduce_add_rmsnorm_gemv_quant(x.unsqueeze(0), r, w, wq, ws, return_quant=True)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_fused_reduce_rejects_bad_slabs(fp8gq, cuda_device):
    K = 4096
    parts = gpu_activation(9, K, 870, cuda_device).view(9, 1, K)
    _, r, w = _norm_inputs(1, K, 871, cuda_device)
    wq, ws = gpu_weight(4096, K, 872, cuda_device)
    with pytest.raises(fp8gq.ShapeError):                 # more slabs than ranks
        fp8gq.fused_reduce_add_rmsnorm_gemv_quant(parts, r, w, wq, ws)
    with pytest.raises(fp8gq.Fp8gqError):                 # residual_out may not alias a slab
        fp8gq.fused_reduce_add_rmsnorm_gemv_quant(parts[:2], r, w, wq, ws, residual_out=parts[1])


# ---------------------------------------- stand-alone SwiGLU writers --

@pytest.mark.parametrize("M, I", [(512, 9728), (16, 9728), (3, 256), (1, 12288)])
def test_swiglu_writers_bit_exact(fp8gq, cuda_device, M, I):
    g = gpu_activation(M, I, 200 + M, cuda_device, std=1.5, outliers=False)
    u = gpu_activation(M, I, 300 + M, cuda_device, std=1.5, outliers=False)
    q, scale = fp8gq.fused_swiglu_quant(g, u)
    y = fp8gq.fused_swiglu(g, u)
    rq, rs, _ = O.swiglu_quant_writer(to_f32(g), to_f32(u))
    assert np.array_equal(to_u8(q), rq)
    assert np.array_equal(to_f32(scale), rs)
    assert np.array_equal(to_f32(y), O.swiglu_writer(to_f32(g), to_f32(u)))


def test_swiglu_writers_on_gate_up_halves(fp8gq, cuda_device):
    """gate and up as the two halves of one gate_up output (row stride 2I)."""
    M, I = 40, 1024
    gu = gpu_activation(M, 2 * I, 17, cuda_device, std=1.5, outliers=False)
    g, u = gu[:, :I], gu[:, I:]
    q, scale = fp8gq.fused_swiglu_quant(g, u)
    rq, rs, _ = O.swiglu_quant_writer(to_f32(g), to_f32(u))
    assert np.array_equal(to_u8(q), rq) and np.array_equal(to_f32(scale), rs)
    out = torch.full((M, I + 64), 7.0, dtype=torch.bfloat16, device=cuda_device)
    fp8gq.fused_swiglu(g, u, out=out[:, :I])
    assert np.array_equal(to_f32(out[:, :I]), O.swiglu_writer(to_f32(g), to_f32(u)))
    assert torch.all(out[:, I:] == 7.0)


@pytest.mark.parametrize("path", WRITER_GOLDEN, ids=[p.stem for p in WRITER_GOLDEN])
def test_swiglu_writer_golden_fixtures(fp8gq, cuda_device, path):
    """The reference's own fused_swiglu / fused_swiglu_quant outputs."""
    d = np.load(path)
    g = bf16_bits_tensor(d["g_bf16"], cuda_device)
    u = bf16_bits_tensor(d["u_bf16"], cuda_device)
    q, scale = fp8gq.fused_swiglu_quant(g, u)
    y = fp8gq.fused_swiglu(g, u)
    assert np.array_equal(to_u8(q), d["q"])
    assert np.array_equal(to_f32(y).view(np.uint32) >> 16, d["y_bf16"].astype(np.uint32))
    assert np.allclose(to_f32(scale), d["scale"], rtol=2.0 ** -22, atol=0.0)


def test_swiglu_writer_stress_battery(fp8gq, cuda_device):
    """benchmarks/stress_tests.py:148-199 on the GPU writers."""
    I = 9728
    g = gpu_activation(8, I, 1, cuda_device, outliers=False)
    u = gpu_activation(8, I, 2, cuda_device, outliers=False)
    q1, s1 = fp8gq.fused_swiglu_quant(g, u)
    q2, s2 = fp8gq.fused_swiglu_quant(g, u)
    assert torch.equal(q1.view(torch.uint8), q2.view(torch.uint8)) and torch.equal(s1, s2)
    z = torch.zeros(4, I, dtype=torch.bfloat16, device=cuda_device)
    q, s = fp8gq.fused_swiglu_quant(z, z)
    assert bool((q.view(torch.uint8) == 0).all()) and bool((s == 1e-30).all())
    t = torch.full((2, I), 20.0, dtype=torch.bfloat16, device=cuda_device)
    q, s = fp8gq.fused_swiglu_quant(t, t)
    assert abs(q.float().abs().max().item() - 448.0) < 1e-2
    n = torch.full((2, I), -50.0, dtype=torch.bfloat16, device=cuda_device)
    out = fp8gq.fused_swiglu(n, u[:2])
    ref = torch.nn.functional.silu(n.float()) * u[:2].float()
    assert bool(torch.isfinite(out).all()) and torch.allclose(out.float(), ref, rtol=1e-2, atol=1e-2)
    g10, u10 = g[:4] * 10, u[:4] * 10
    q, s = fp8gq.fused_swiglu_quant(g10, u10)
    y = torch.nn.functional.silu(g10.float()) * u10.float()
    am = y.abs().view(4, -1, 128).amax(-1)
    ns = (am / 448.0).clamp_min(1e-30)
    nq = (y.view(4, -1, 128) / ns.unsqueeze(-1)).clamp(-448, 448).view(4, -1).to(torch.float8_e4m3fn)
    assert (q.view(torch.uint8) == nq.view(torch.uint8)).float().mean().item() > 0.999


# ------------------------------------------ launch ordering (PDL) --------

@pytest.mark.parametrize("static_weights", [False, True])
@pytest.mark.parametrize("M, kernel", [(1, "row"), (1, "tm"), (4, "tm")])
def test_chained_linears_see_their_producer(fp8gq, cuda_device, static_weights, M, kernel):
    """out1 = lin1(x); out2 = lin2(out1) back to back on one stream, eager and
    in a CUDA graph: the second kernel may start early (programmatic dependent
    launch) but must read out1 only after the first has finished."""
    K1, N1, N2 = 2048, 4096, 2560
    x = gpu_activation(M, K1, 110, cuda_device)
    w1, s1 = gpu_weight(N1, K1, 111, cuda_device)
    w2, s2 = gpu_weight(N2, N1, 112, cuda_device)
    ref1 = fp8gq.fused_gemv_quant(x, w1, s1, kernel=kernel)
    torch.cuda.synchronize()
    ref2 = fp8gq.fused_gemv_quant(ref1, w2, s2, kernel=kernel)
    torch.cuda.synchronize()
    prev = fp8gq.set_static_weights(static_weights)
    try:
        out1 = torch.empty_like(ref1)
        out2 = torch.empty_like(ref2)
        for _ in range(3):
            out1.zero_()
            out2.zero_()
            fp8gq.fused_gemv_quant(x, w1, s1, out=out1, kernel=kernel)
            fp8gq.fused_gemv_quant(out1, w2, s2, out=out2, kernel=kernel)
        torch.cuda.synchronize()
        assert torch.equal(out1, ref1) and torch.equal(out2, ref2)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fp8gq.fused_gemv_quant(x, w1, s1, out=out1, kernel=kernel)
            fp8gq.fused_gemv_quant(out1, w2, s2, out=out2, kernel=kernel)
        for _ in range(3):
            out1.zero_()
            out2.zero_()
            g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out1, ref1) and torch.equal(out2, ref2)
        del g
    finally:
        fp8gq.set_static_weights(prev)


# ------------------------------------------------------- the patch layer --

def test_patch_wrappers_on_gpu(fp8gq, cuda_device):
    import types
    import fp8gq.patch_fp8_fused_tail as P
    calls = []
    mod = types.ModuleType("fp8_utils")
    mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback = lambda *a: calls.append(a) or None
    P.install(mod)
    try:
        K, N = 4096, 6144
        wq, ws = gpu_weight(N, K, 70, cuda_device)
        for M in (1, 4):
            x = gpu_activation(M, K, 71, cuda_device).view(M, 1, K)
            bias = torch.randn(N, device=cuda_device).bfloat16()
            out = mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback(
                input=x, weight=wq, block_size=[128, 128], weight_scale=ws, input_scale=None, bias=bias)
            assert out.shape == (M, 1, N)
            want = fp8gq.fused_gemv_quant(x.view(M, K), wq, ws) + bias
            assert torch.equal(out.view(M, N), want)
        assert not calls
        # routed sizes whose activation the kernels cannot read in place (rows
        # starting 8 bytes in; every other element along K) still take the
        # fused path, through an aligned copy, and match the oracle
        for M, step in ((1, 1), (4, 1), (3, 2)):
            x = gpu_activation(M, K, 73 + M, cuda_device)
            base = torch.zeros(M * K * step + 64, dtype=torch.bfloat16, device=cuda_device)
            xv = base[4:4 + M * K * step].view(M, K * step)[:, ::step]
            xv.copy_(x)
            assert xv.data_ptr() % 16 != 0 or xv.stride(1) != 1
            out = mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback(xv, wq, [128, 128], ws, None, None)
            assert torch.equal(out, fp8gq.fused_gemv_quant(x, wq, ws))
            _, exact, _, _ = oracle_of(x, wq, ws)
            assert_close(to_f32(out), exact, 3.0)
        assert not calls
        x = gpu_activation(32, K, 72, cuda_device)
        mod.flashinfer_gemm_w8a8_block_fp8_linear_with_fallback(x, wq, [128, 128], ws, None, None)
        assert len(calls) == 1
    finally:
        P.uninstall(mod)


def test_misaligned_activation_raises(fp8gq, cuda_device):
    wq, ws = gpu_weight(256, 256, 80, cuda_device)
    x = torch.zeros(1, 264, dtype=torch.bfloat16, device=cuda_device)[:, 4:260]
    with pytest.raises(fp8gq.Fp8gqError) as e:
        fp8gq.fused_gemv_quant(x, wq, ws)
    assert e.value.status == 3


def test_no_device_error_recorded(fp8gq, cuda_device):
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
