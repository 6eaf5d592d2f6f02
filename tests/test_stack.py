"""Stack runner (fp8gq_stack_prepare / fp8gq_stack_run): a list of linears in
one persistent launch.

CPU: the dependency analysis of fp8gq_stack_dependencies on made-up
addresses (no device is touched) and argument checks.
GPU: every linear's output against the oracle applied to that linear's own
input as the GPU left it (chained lists, SwiGLU, M from 1 to 16, lists whose
linears have fewer tiles than the grid has CTAs, buffer reuse), runs repeated
bit for bit, and the Qwen3-8B decode layer at full size."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import assert_close, to_f32, to_u8


def _lib():
    from fp8gq import _lib
    return _lib


def fake(x, K, w, N, out, ldx=None, ldo=None, swiglu=0):
    L = _lib().StackLinear()
    L.x, L.ldx = x, ldx if ldx is not None else (2 * K if swiglu else K)
    L.w, L.ldw = w, K
    L.ws, L.ldws = w + (1 << 24), K // 128
    L.out, L.ldo = out, ldo if ldo is not None else N
    L.N, L.K, L.swiglu, L.reserved = N, K, swiglu, 0
    return L


def deps(lins, M=1):
    lib = _lib().load()
    arr = (_lib().StackLinear * len(lins))(*lins)
    dep = (ctypes.c_int * len(lins))()
    st = lib.fp8gq_stack_dependencies(arr, len(lins), M, dep)
    return st, list(dep)


A, B, C, D = (1 << 32), (2 << 32), (3 << 32), (4 << 32)
W = 8 << 32


def test_dependencies_of_a_chain():
    # qkv -> o (first 4096 columns of qkv's output) -> gate_up -> down (SwiGLU)
    lins = [fake(A, 4096, W, 6144, B), fake(B, 4096, W + (1 << 28), 4096, C, ldx=6144),
            fake(C, 4096, W + (2 << 28), 24576, D), fake(D, 12288, W + (3 << 28), 4096, A, swiglu=1)]
    assert deps(lins) == (0, [-1, 0, 1, 2])


def test_independent_linears_do_not_wait():
    lins = [fake(A + i * (1 << 20), 4096, W, 4096, B + i * (1 << 20)) for i in range(4)]
    assert deps(lins) == (0, [-1, -1, -1, -1])


def test_write_after_read_and_write_after_write_wait():
    # linear 2 overwrites linear 0's input; linear 3 writes linear 1's output again
    lins = [fake(A, 256, W, 256, B), fake(C, 256, W, 256, D), fake(C + 4096, 256, W, 256, A + 256),
            fake(B + (1 << 20), 256, W, 256, D + 128)]
    assert deps(lins) == (0, [-1, -1, 0, 1])


def test_the_latest_conflict_is_chosen_and_ranges_use_rows():
    # M = 4 rows with a row stride of 1024 elements: row 3 of linear 0's output
    # reaches into the input of linear 2; linear 1 does not touch either
    lins = [fake(A, 128, W, 128, B, ldo=1024), fake(C, 128, W, 128, D), fake(B + 3 * 2048, 128, W, 128, C + (1 << 20))]
    assert deps(lins, M=4) == (0, [-1, -1, 0])
    assert deps(lins, M=1) == (0, [-1, -1, -1])   # one row: linear 0 writes only B .. B + 256


def test_argument_checks():
    ok = fake(A, 256, W, 256, B)
    assert deps([ok], M=17)[0] == 2                               # at most 16 tokens
    assert deps([ok], M=0)[0] == 2
    assert deps([fake(A, 200, W, 256, B)])[0] == 2                 # K not a multiple of 128
    assert deps([fake(A, 256, W, 256, B, ldx=128)])[0] == 4        # ldx < K
    assert deps([fake(A, 256, W, 256, B, ldx=260)])[0] == 3        # rows not 16-byte aligned
    assert deps([fake(A, 256, W, 256, B, ldx=256, swiglu=1)])[0] == 4   # SwiGLU input needs 2K columns
    assert deps([fake(A + 8, 256, W, 256, B)])[0] == 3
    bad = fake(A, 256, W, 256, B)
    bad.reserved = 1
    assert deps([bad])[0] == 8
    lib = _lib().load()
    assert lib.fp8gq_stack_dependencies(None, 1, 1, (ctypes.c_int * 1)()) == 1
    assert lib.fp8gq_stack_run(None, None) == 1


def test_python_list_checks():
    import fp8gq
    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    w = torch.zeros(256, 256, dtype=torch.float8_e4m3fn)
    s = torch.ones(2, 2)
    o = torch.zeros(1, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fp8gq.StackRunner([fp8gq.Linear(x, w, s, o)])
    from fp8gq import stack
    with pytest.raises(fp8gq.ShapeError):
        stack._array([fp8gq.Linear(torch.zeros(17, 256, dtype=torch.bfloat16), w, s,
                                   torch.zeros(17, 256, dtype=torch.bfloat16))])
    with pytest.raises(fp8gq.ShapeError):
        stack._array([fp8gq.Linear(x, w, s, o, swiglu=True)])


# ------------------------------------------------------------------ GPU --
def gpu_weight(N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0
    q = (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K)
    return q.contiguous(), ws.contiguous()


def gpu_activation(M, K, seed, dev, std=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev) * std
    ch = torch.randperm(K, generator=g, device=dev)[: max(1, round(0.01 * K))]
    x[:, ch] *= 20.0
    return x.bfloat16().contiguous()


def check_each(lins, inputs, ulps=3):
    """Every linear's output against the oracle applied to the input it read
    (``inputs[l]``, a CPU copy taken where a later linear overwrites it)."""
    for l, lin in enumerate(lins):
        fn = O.fused_swiglu_q_gemm if lin.swiglu else O.fused_gemv_quant
        _, exact, _, _ = fn(inputs[l], to_u8(lin.w), to_f32(lin.ws))
        try:
            assert_close(to_f32(lin.out), exact, ulps)
        except AssertionError as e:
            raise AssertionError(f"linear {l}: {e}") from None


def decoder_chain(M, dims, dev, seed=0):
    """qkv -> o -> gate_up -> down(SwiGLU) -> next qkv ... with the dims of
    (hidden H, qkv width Q, intermediate I) for each layer; o reads the first
    H columns of qkv's output (an attention stand-in)."""
    import fp8gq
    H, Q, I = dims["H"], dims["Q"], dims["I"]
    layers = dims["layers"]
    h = gpu_activation(M, H, seed, dev)
    lins = []
    x = h
    for L in range(layers):
        s = seed + 100 * L
        qkv = torch.empty(M, Q, dtype=torch.bfloat16, device=dev)
        lins.append(fp8gq.Linear(x, *gpu_weight(Q, H, s + 1, dev), qkv))
        o = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        lins.append(fp8gq.Linear(qkv[:, :H], *gpu_weight(H, H, s + 2, dev), o))
        gu = torch.empty(M, 2 * I, dtype=torch.bfloat16, device=dev)
        lins.append(fp8gq.Linear(o, *gpu_weight(2 * I, H, s + 3, dev), gu))
        d = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        lins.append(fp8gq.Linear(gu, *gpu_weight(H, I, s + 4, dev), d, swiglu=True))
        x = d
    return lins


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 2, 5, 16])
def test_decoder_chain_matches_oracle(cuda_device, M):
    import fp8gq
    dev = cuda_device
    lins = decoder_chain(M, {"H": 512, "Q": 768, "I": 1024, "layers": 3}, dev, seed=M)
    runner = fp8gq.StackRunner(lins)
    assert runner.dependencies == [-1] + list(range(len(lins) - 1))
    runner.run()
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    check_each(lins, [to_f32(lin.x) for lin in lins])


@pytest.mark.gpu
def test_runs_repeat_bit_for_bit_and_match_the_tile_kernel(cuda_device):
    import fp8gq
    dev = cuda_device
    lins = decoder_chain(1, {"H": 1024, "Q": 1536, "I": 2048, "layers": 2}, dev, seed=7)
    runner = fp8gq.StackRunner(lins)
    runner.run()
    first = [lin.out.clone() for lin in lins]
    for _ in range(3):
        for lin in lins:
            lin.out.zero_()
        runner.run()
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    for a, lin in zip(first, lins):
        assert torch.equal(a, lin.out)
    # the per-linear tile kernel on the same inputs: same quantised bytes,
    # outputs within the accumulation-order tolerance of each other
    for lin in lins:
        op = fp8gq.fused_swiglu_q_gemm if lin.swiglu else fp8gq.fused_gemv_quant
        kw = {} if lin.swiglu else {"kernel": "tm"}
        ref = op(lin.x, lin.w, lin.ws, **kw)
        _, exact, _, _ = (O.fused_swiglu_q_gemm if lin.swiglu else O.fused_gemv_quant)(
            to_f32(lin.x), to_u8(lin.w), to_f32(lin.ws))
        assert_close(to_f32(ref), exact, 3)
        assert_close(to_f32(lin.out), exact, 3)


@pytest.mark.gpu
def test_small_linears_leave_most_ctas_idle(cuda_device):
    """One-tile linears (N = K = 128): a single CTA works, the others only
    count themselves done; plus a linear with more row blocks than CTAs."""
    import fp8gq
    dev = cuda_device
    lins = []
    x = gpu_activation(3, 128, 1, dev)
    for i in range(5):
        out = torch.empty(3, 128, dtype=torch.bfloat16, device=dev)
        lins.append(fp8gq.Linear(x, *gpu_weight(128, 128, 10 + i, dev), out))
        x = out
    big = torch.empty(3, 160 * 128, dtype=torch.bfloat16, device=dev)
    lins.append(fp8gq.Linear(x, *gpu_weight(160 * 128, 128, 20, dev), big))
    runner = fp8gq.StackRunner(lins)
    runner.run()
    runner.run()
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    check_each(lins, [to_f32(lin.x) for lin in lins])


@pytest.mark.gpu
def test_buffer_reuse_waits(cuda_device):
    """Linear 1 overwrites linear 0's input and linear 2 reads it again: the
    first must have read the original, the last the new contents."""
    import fp8gq
    dev = cuda_device
    a = gpu_activation(2, 1024, 3, dev)
    a0 = to_f32(a)
    b = torch.empty(2, 1024, dtype=torch.bfloat16, device=dev)
    c = torch.empty(2, 1024, dtype=torch.bfloat16, device=dev)
    x1 = gpu_activation(2, 2048, 4, dev)
    lins = [fp8gq.Linear(a, *gpu_weight(1024, 1024, 5, dev), b),
            fp8gq.Linear(x1, *gpu_weight(1024, 2048, 6, dev), a),
            fp8gq.Linear(a, *gpu_weight(1024, 1024, 7, dev), c)]
    runner = fp8gq.StackRunner(lins)
    assert runner.dependencies == [-1, 0, 1]
    runner.run()
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    check_each(lins, [a0, to_f32(x1), to_f32(a)])


@pytest.mark.gpu
def test_qwen3_8b_decode_layers_full_size(cuda_device):
    """Two layers of the Qwen3-8B decode linears at M = 1 (qkv 4096->6144,
    o 4096->4096, gate_up 4096->24576, down 12288->4096 with SwiGLU),
    captured in a CUDA graph and replayed."""
    import fp8gq
    dev = cuda_device
    lins = decoder_chain(1, {"H": 4096, "Q": 6144, "I": 12288, "layers": 2}, dev, seed=11)
    runner = fp8gq.StackRunner(lins)
    runner.run()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        runner.run()
    for lin in lins:
        lin.out.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    check_each(lins, [to_f32(lin.x) for lin in lins])
    del g
