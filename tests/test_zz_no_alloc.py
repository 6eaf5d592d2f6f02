"""fp8gq_gemv_quant_tm_noalloc through the C ABI.

This entry point serves callers that cannot allocate device memory when they
call the library -- a server that has already handed nearly all HBM to its own
pool, a decode loop that cannot pay for cudaMalloc's implicit synchronisation,
a C caller with no allocator to make a zeroed workspace.  Instead of a
caller-provided workspace it uses a fixed 8 MiB device array inside the
library, so it must agree with the workspace entry point (fp8gq_gemv_quant_tm)
on every shape that fits, call after call, while the array keeps whatever the
previous call left in it; shapes that do not fit must be refused.

The array holds the split-K counters and partial sums and, for the
pre-quantised activation feed, the quantised activation.  The auto choice
reduces most split-K partial sums inside thread-block clusters, so two cases
force the other strategies (fp8gq_set_tm_options) to make the array carry the
data: the split-K hand-off through memory, and the pre-quantised feed.  Each
alternates two shapes with different row-block counts and splits on one
stream, so leftover counters and partial sums of one shape meet the next.

The file is named to be collected last; it needs nothing from other tests and
passes when run on its own in a fresh process.
"""
import numpy as np
import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import assert_close, to_f32

pytestmark = pytest.mark.gpu


def _operands(M, K, N, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = (torch.randn(M, K, generator=g, device=dev)).bfloat16()
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = (blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0).contiguous()
    wq = (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K).contiguous()
    return x, wq, ws


def _call_noalloc(lib, x, wq, ws, out):
    M, K = x.shape
    N = wq.shape[0]
    return lib.fp8gq_gemv_quant_tm_noalloc(
        x.data_ptr(), x.stride(0), wq.data_ptr(), wq.stride(0), ws.data_ptr(), ws.stride(0),
        out.data_ptr(), out.stride(0), M, N, K, None, None, torch.cuda.current_stream().cuda_stream)


def _call_workspace(lib, x, wq, ws, out):
    M, K = x.shape
    N = wq.shape[0]
    nbytes = lib.fp8gq_workspace_bytes(max(M, 2), N, K)
    work = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
    st = lib.fp8gq_gemv_quant_tm(
        x.data_ptr(), x.stride(0), wq.data_ptr(), wq.stride(0), ws.data_ptr(), ws.stride(0),
        out.data_ptr(), out.stride(0), M, N, K, None, None, work.data_ptr(), nbytes,
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return st


@pytest.fixture(scope="module")
def lib(cuda_device):
    from fp8gq import _lib
    return _lib.load()


@pytest.mark.parametrize("M, K, N", [(4, 4096, 6144), (16, 2560, 19456), (1, 12288, 4096)])
def test_noalloc_matches_workspace_entry_point_twice(lib, cuda_device, M, K, N):
    x, wq, ws = _operands(M, K, N, seed=M + K + N, dev=cuda_device)
    ref = torch.empty(M, N, dtype=torch.bfloat16, device=cuda_device)
    assert _call_workspace(lib, x, wq, ws, ref) == 0
    exact = O.fused_gemv_quant(to_f32(x), wq.cpu().view(torch.uint8).numpy(), to_f32(ws))[1]
    for call in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        st = _call_noalloc(lib, x, wq, ws, out)
        assert st == 0, lib.fp8gq_status_string(st)
        torch.cuda.synchronize()
        # the tolerance the other tile-kernel tests use, against the workspace
        # entry point and against the oracle
        assert_close(to_f32(out), to_f32(ref).astype(np.float64), 3.0)
        assert_close(to_f32(out), exact, 3.0)


# two shapes with different row-block counts and splits: (M, K, N)
ALTERNATING = [(1, 12288, 4096), (4, 4096, 6144)]


@pytest.mark.parametrize("option", ["workspace_splitk", "prequant"])
def test_noalloc_scratch_carries_the_data_across_alternating_shapes(lib, cuda_device, option):
    import fp8gq
    flags = {"workspace_splitk": fp8gq.TM_WORKSPACE_SPLITK,
             "prequant": fp8gq.TM_PREQUANT_ACTIVATIONS | fp8gq.TM_WORKSPACE_SPLITK}[option]
    ops = [_operands(M, K, N, seed=100 + i, dev=cuda_device) for i, (M, K, N) in enumerate(ALTERNATING)]
    prev = fp8gq.set_tm_options(flags)
    try:
        refs = []
        for x, wq, ws in ops:
            ref = torch.empty(x.shape[0], wq.shape[0], dtype=torch.bfloat16, device=cuda_device)
            assert _call_workspace(lib, x, wq, ws, ref) == 0
            refs.append(ref)
        # A, B, A, B, A, B on one stream with no synchronisation in between:
        # every call starts on the counters and partial sums the last one left
        outs = []
        for rep in range(3):
            for i, (x, wq, ws) in enumerate(ops):
                out = torch.full((x.shape[0], wq.shape[0]), float("nan"), dtype=torch.bfloat16,
                                 device=cuda_device)
                st = _call_noalloc(lib, x, wq, ws, out)
                assert st == 0, lib.fp8gq_status_string(st)
                outs.append((i, out))
        torch.cuda.synchronize()
    finally:
        fp8gq.set_tm_options(prev)
    assert fp8gq.device_error() == 0
    # same grid, same products, same order of additions: bit-identical to the
    # workspace entry point under the same options, and within the tile
    # kernel's tolerance of the oracle
    for i, out in outs:
        assert torch.equal(out, refs[i]), f"shape {ALTERNATING[i]}: differs from the workspace entry point"
    for i, (x, wq, ws) in enumerate(ops):
        exact = O.fused_gemv_quant(to_f32(x), wq.cpu().view(torch.uint8).numpy(), to_f32(ws))[1]
        assert_close(to_f32(refs[i]), exact, 3.0)


def test_noalloc_refuses_shapes_beyond_its_scratch(lib, cuda_device):
    # M = 64 needs 64-token partial sums for every CTA: more than 8 MiB
    x, wq, ws = _operands(64, 1024, 2048, seed=5, dev=cuda_device)
    out = torch.empty(64, 2048, dtype=torch.bfloat16, device=cuda_device)
    assert _call_noalloc(lib, x, wq, ws, out) == 10          # FP8GQ_ERR_SCRATCH_LIMIT
    assert b"8 MiB" in lib.fp8gq_status_string(10)
