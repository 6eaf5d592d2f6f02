"""The bounded waits give up, report, and leave the GPU usable.

The reference's only failure mechanism is a catch-all that swallows any error
of the fused call and reruns the original linear
(patches/patch_fp8_fused_tail.py:16-26).  Here a routed call never falls back;
the failure that can strand a kernel is a lost peer GPU in an N-sharded step,
whose flag never rises.  Every such wait is bounded: it gives up after the
peer limit, records the site in the device error word, and the kernel runs to
its end.  These tests make that happen on one GPU, without a fault: the
gathered call's "peer" is a second local buffer and flag array that nothing
ever raises.  They check that the call ends within about the limit, that the
error word names the gather wait, and that after the word is cleared an
ordinary call on the same context passes parity.
"""
import ctypes
import time

import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import assert_close, to_f32, to_u8

pytestmark = pytest.mark.gpu

LIMIT_NS = 200_000_000          # 200 ms: the peer limit set for these tests
SITE_GATHER = 0x80000000 | 8    # error word of a gather wait that gave up


@pytest.fixture(scope="module")
def fp8gq(cuda_device):
    import fp8gq as mod
    mod.load()
    return mod


def _operands(M, K, N, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev).bfloat16()
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = (blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0).contiguous()
    wq = (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K).contiguous()
    return x, wq, ws


class _LonePeer:
    """A two-rank gather descriptor for rank 0 whose rank-1 buffers are local
    stand-ins.  The state says one gathered call has already happened (this
    rank's sequence number is 1 and its own flag is raised) while the peer's
    flag stays 0, as if rank 1 had died after that call."""

    def __init__(self, fp8gq, M, N, dev):
        from fp8gq import _lib
        self.full = [torch.zeros(M, 2 * N, dtype=torch.bfloat16, device=dev) for _ in range(2)]
        self.flags = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)     # counter, seq
        self.state[1] = 1
        self.flags[0][0] = 1
        g = _lib.Gather()
        for r in range(2):
            g.out[r] = self.full[r].data_ptr()
            g.flags[r] = self.flags[r].data_ptr()
        g.counter = self.state.data_ptr()
        g.seq = self.state.data_ptr() + 4
        g.ldo = 2 * N
        g.col0 = 0
        g.world = 2
        g.rank = 0
        g.wait_input = 1
        g.local_out = 0
        self.desc = g


@pytest.fixture
def short_limit(fp8gq):
    torch.cuda.synchronize()
    fp8gq.device_error(clear=True)
    prev = fp8gq.set_wait_limit_ns(LIMIT_NS)
    yield
    torch.cuda.synchronize()
    fp8gq.set_wait_limit_ns(prev)
    fp8gq.device_error(clear=True)


def _timed(fn):
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = fn()
    torch.cuda.synchronize()
    return st, time.perf_counter() - t0


# (M, K, N): the row kernel (M == 1, small weight) and the tile kernel (M = 4)
@pytest.mark.parametrize("M, K, N", [(1, 4096, 1024), (4, 2048, 1024)])
def test_gathered_call_gives_up_on_a_silent_peer(fp8gq, cuda_device, short_limit, M, K, N):
    from fp8gq import _lib, ops
    lib = _lib.load()
    x, wq, ws = _operands(M, K, N, seed=M * 7 + 1, dev=cuda_device)
    peer = _LonePeer(fp8gq, M, N, cuda_device)
    nbytes = lib.fp8gq_workspace_bytes(M, N, K)
    work = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=cuda_device)
    stream = ops._stream(cuda_device)

    def call():
        return lib.fp8gq_fused_gemv_quant_gather(
            x.data_ptr(), x.stride(0), wq.data_ptr(), wq.stride(0), ws.data_ptr(), ws.stride(0), M, N, K,
            ctypes.byref(peer.desc), work.data_ptr() if nbytes else None, nbytes, stream)

    st, dt = _timed(call)
    assert st == 0, lib.fp8gq_status_string(st)
    # the call waited for the whole limit and no more than the in-kernel
    # waits' limit behind it
    assert 0.8 * LIMIT_NS * 1e-9 <= dt < 2.0 * LIMIT_NS * 1e-9 + 0.5, f"call took {dt:.3f} s"
    assert fp8gq.device_error() == SITE_GATHER, hex(fp8gq.device_error())

    # fp8gq_gather_wait on the same silent peer gives up the same way
    fp8gq.device_error(clear=True)
    st, dt = _timed(lambda: lib.fp8gq_gather_wait(ctypes.byref(peer.desc), stream))
    assert st == 0, lib.fp8gq_status_string(st)
    assert 0.8 * LIMIT_NS * 1e-9 <= dt < 2.0 * LIMIT_NS * 1e-9 + 0.5, f"wait took {dt:.3f} s"
    assert fp8gq.device_error() == SITE_GATHER, hex(fp8gq.device_error())

    # after clearing the word the context is usable: an ordinary call passes
    # parity against the oracle
    fp8gq.device_error(clear=True)
    out, xq, sx = fp8gq.fused_gemv_quant(x, wq, ws, return_quant=True)
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    _, exact, rq, rs = O.fused_gemv_quant(to_f32(x), to_u8(wq), to_f32(ws))
    assert (to_u8(xq) == rq).all() and (to_f32(sx) == rs).all()
    assert_close(to_f32(out), exact, 3.0)


def test_wait_limit_range_is_checked(fp8gq):
    from fp8gq import _lib
    with pytest.raises(_lib.Fp8gqError):
        fp8gq.set_wait_limit_ns(10)                 # below 1 ms
    with pytest.raises(_lib.Fp8gqError):
        fp8gq.set_wait_limit_ns(60 * 10**9)         # above 20 s
    prev = fp8gq.set_wait_limit_ns(2 * 10**9)
    assert fp8gq.set_wait_limit_ns(prev) == 2 * 10**9
