"""Tagged-word gather (fp8gq_gather.tagged) on one GPU.

Every stored word of a tagged output carries two bf16 columns and the
sequence number of the call that wrote it; a call that reads such an output
polls the words it reads instead of waiting for a flag.  These tests drive
the protocol with a two-rank descriptor for rank 0 whose rank-1 buffers are
local stand-ins.  Rank 1's slice of each input is written, with the right
tag, by the host before the call that reads it (stream order), so no kernel
ever waits for another kernel.  A chain of three calls covers the tile
kernel and the row kernel (one and four rows per group) as producers and as
consumers, the SwiGLU consumer and fp8gq_gather_decode; each output slice
must equal, bit for bit, the plain single-GPU op on the same full input, and
carry its call's sequence number on both ranks' buffers.  The bounded waits
of the protocol -- a consumer's word poll, the decode kernel, and a
publishing call's wait for the ranks' own flag slots -- give up on a silent
peer after the limit with the gather site in the error word.
"""
import ctypes
import time

import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import assert_close, to_f32, to_u8

from fp8gq.dist import tags, untag

pytestmark = pytest.mark.gpu

LIMIT_NS = 200_000_000          # 200 ms: the peer limit set for the timeout tests
SITE_GATHER = 0x80000000 | 8    # error word of a gather wait that gave up


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
    wq = (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K).contiguous()
    return wq, ws


def _tagged(values: torch.Tensor, tag: int) -> torch.Tensor:
    """bf16 [M, n] -> tagged words [M, n/2] (int64) carrying `tag`."""
    lo = values.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return lo | (tag << 32)


class _Pair:
    """Rank 0 of a two-rank tagged gather whose rank-1 buffers are local."""

    def __init__(self, dev):
        self.dev = dev
        self.flags = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
        self.state = torch.zeros(2, dtype=torch.int32, device=dev)     # counter, seq

    def words(self, M, N):
        """Rank 0's and rank 1's buffers of one tagged [M, N] output."""
        return [torch.zeros(M, N // 2, dtype=torch.int64, device=self.dev) for _ in range(2)]

    def desc(self, bufs, wait_input):
        from fp8gq import _lib
        g = _lib.Gather()
        for r in range(2):
            g.out[r] = bufs[r].data_ptr()
            g.flags[r] = self.flags[r].data_ptr()
        g.counter = self.state.data_ptr()
        g.seq = self.state.data_ptr() + 4
        g.ldo = 2 * bufs[0].stride(0)
        g.col0 = 0
        g.world = 2
        g.rank = 0
        g.wait_input = 1 if wait_input else 0
        g.local_out = 0
        g.tagged = 1
        return g


def _call(fn_name, x_ptr, ldx, wq, ws, M, N, K, desc, dev):
    from fp8gq import _lib, ops
    lib = _lib.load()
    nbytes = lib.fp8gq_workspace_bytes(M, N, K)
    work = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)
    st = getattr(lib, fn_name)(x_ptr, ldx, wq.data_ptr(), wq.stride(0), ws.data_ptr(), ws.stride(0), M, N, K,
                               ctypes.byref(desc), work.data_ptr() if nbytes else None, nbytes, ops._stream(dev))
    torch.cuda.synchronize()
    assert st == 0, lib.fp8gq_status_string(st)


# (M, K1, N1, N2, N3): call 1 x [M, K1] -> tagged [M, N1]; call 2 reads it
# (wait_input) -> tagged [M, N2]; call 3 (SwiGLU, I = N2 / 2) reads that ->
# tagged [M, N3]; rank 0 holds the first half of each output's columns.
CASES = [
    # M = 1: call 1 on the tile kernel (6144 x 4096 slice, 25 MB), call 2 on
    # the row kernel with one row per group (K = 12288), call 3 on the row
    # kernel's SwiGLU form (four rows per group)
    (1, 4096, 12288, 2048, 1024),
    # M = 4: the tile kernel throughout (resident tagged feed)
    (4, 2048, 2048, 2048, 1024),
]


@pytest.mark.parametrize("M, K1, N1, N2, N3", CASES)
def test_tagged_chain_matches_the_plain_op(fp8gq, cuda_device, M, K1, N1, N2, N3):
    dev = cuda_device
    torch.cuda.synchronize()
    fp8gq.device_error(clear=True)
    g = torch.Generator(device=dev).manual_seed(M * 100 + 3)
    x = torch.randn(M, K1, generator=g, device=dev).bfloat16()
    pair = _Pair(dev)
    w1 = [_weight(N1 // 2, K1, 11 + r, dev) for r in range(2)]
    w2 = [_weight(N2 // 2, N1, 21 + r, dev) for r in range(2)]
    w3 = [_weight(N3 // 2, N2 // 2, 31 + r, dev) for r in range(2)]
    o1, o2, o3 = pair.words(M, N1), pair.words(M, N2), pair.words(M, N3)

    def check_slice(bufs, plain, tag, N):
        own = bufs[0][:, :N // 4]
        assert torch.equal(own, bufs[1][:, :N // 4]), "the slice must land in every rank's buffer"
        assert bool((tags(own) == tag).all()), "every own word carries its call's sequence number"
        assert torch.equal(untag(own), plain), "tagged values must equal the plain op bit for bit"

    def fill_peer(bufs, values, tag, N):
        bufs[0][:, N // 4:] = _tagged(values, tag)

    # call 1: bf16 input, publishing without an input wait (sequence 1)
    _call("fp8gq_fused_gemv_quant_gather", x.data_ptr(), x.stride(0), w1[0][0], w1[0][1], M, N1 // 2, K1,
          pair.desc(o1, False), dev)
    full1 = torch.cat([fp8gq.fused_gemv_quant(x, *w1[r]) for r in range(2)], dim=1)
    check_slice(o1, full1[:, :N1 // 2], 1, N1)
    fill_peer(o1, full1[:, N1 // 2:], 1, N1)

    # call 2: reads call 1's words (sequence 2)
    _call("fp8gq_fused_gemv_quant_gather", o1[0].data_ptr(), 2 * o1[0].stride(0), w2[0][0], w2[0][1], M,
          N2 // 2, N1, pair.desc(o2, True), dev)
    full2 = torch.cat([fp8gq.fused_gemv_quant(full1, *w2[r]) for r in range(2)], dim=1)
    check_slice(o2, full2[:, :N2 // 2], 2, N2)
    fill_peer(o2, full2[:, N2 // 2:], 2, N2)
    _, exact, _, _ = O.fused_gemv_quant(to_f32(full1), to_u8(w2[0][0]), to_f32(w2[0][1]))
    assert_close(to_f32(untag(o2[0][:, :N2 // 4])), exact, 3.0)

    # call 3: SwiGLU of call 2's words [gate | up] (sequence 3)
    _call("fp8gq_fused_swiglu_q_gemm_gather", o2[0].data_ptr(), 2 * o2[0].stride(0), w3[0][0], w3[0][1], M,
          N3 // 2, N2 // 2, pair.desc(o3, True), dev)
    full3 = torch.cat([fp8gq.fused_swiglu_q_gemm(full2, *w3[r]) for r in range(2)], dim=1)
    check_slice(o3, full3[:, :N3 // 2], 3, N3)
    fill_peer(o3, full3[:, N3 // 2:], 3, N3)

    # decode: the full tagged output as bf16
    from fp8gq import _lib, ops
    lib = _lib.load()
    dst = torch.full((M, N3), float("nan"), dtype=torch.bfloat16, device=dev)
    st = lib.fp8gq_gather_decode(ctypes.byref(pair.desc(o3, True)), M, N3, dst.data_ptr(), dst.stride(0),
                                 ops._stream(dev))
    torch.cuda.synchronize()
    assert st == 0, lib.fp8gq_status_string(st)
    assert torch.equal(dst, full3)
    assert int(pair.state[1]) == 3 and int(pair.flags[0][0]) == 3, "sequence and own flag slot advance"
    assert int(pair.state[0]) == 0, "the CTA counter is reset"
    assert fp8gq.device_error() == 0


def test_tagged_argument_checks(fp8gq, cuda_device):
    """Tagged calls reject what the protocol cannot carry."""
    from fp8gq import _lib, ops
    lib = _lib.load()
    CODE = {v: k for k, v in _lib.STATUS.items()}
    dev = cuda_device
    pair = _Pair(dev)
    x = torch.randn(32, 2048, device=dev).bfloat16()
    wq, ws = _weight(1024, 2048, 5, dev)
    o = pair.words(32, 2048)
    nbytes = lib.fp8gq_workspace_bytes(32, 1024, 2048)
    work = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)

    def status(M, desc, xp=None, ldx=2048):
        return lib.fp8gq_fused_gemv_quant_gather(xp or x.data_ptr(), ldx, wq.data_ptr(), 2048, ws.data_ptr(), 16,
                                                 M, 1024, 2048, ctypes.byref(desc), work.data_ptr(), nbytes,
                                                 ops._stream(dev))
    # M > 16: more than one launch per call
    assert status(32, pair.desc(o, False)) == CODE["FP8GQ_ERR_UNSUPPORTED"]
    # a waited-for input must be 16-byte aligned words
    assert status(1, pair.desc(o, True), xp=o[0].data_ptr() + 8) == CODE["FP8GQ_ERR_ALIGNMENT"]
    # odd column offset
    d = pair.desc(o, False)
    d.col0 = 1
    assert status(1, d) == CODE["FP8GQ_ERR_ALIGNMENT"]
    # flags-only entry points
    assert lib.fp8gq_gather_wait(ctypes.byref(pair.desc(o, True)), ops._stream(dev)) == \
        CODE["FP8GQ_ERR_UNSUPPORTED"]
    d = pair.desc(o, True)
    d.tagged = 0
    dst = torch.empty(1, 2048, dtype=torch.bfloat16, device=dev)
    assert lib.fp8gq_gather_decode(ctypes.byref(d), 1, 2048, dst.data_ptr(), 2048, ops._stream(dev)) == \
        CODE["FP8GQ_ERR_UNSUPPORTED"]
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0


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


def _gave_up(fp8gq, lib, st, dt):
    assert st == 0, lib.fp8gq_status_string(st)
    assert 0.8 * LIMIT_NS * 1e-9 <= dt < 2.0 * LIMIT_NS * 1e-9 + 0.5, f"call took {dt:.3f} s"
    assert fp8gq.device_error() == SITE_GATHER, hex(fp8gq.device_error())
    fp8gq.device_error(clear=True)


# the row kernel (M == 1, small weight) and the tile kernel (M = 4)
@pytest.mark.parametrize("M, K, N", [(1, 4096, 1024), (4, 2048, 1024)])
def test_tagged_waits_give_up_on_a_silent_peer(fp8gq, cuda_device, short_limit, M, K, N):
    """A peer whose words never arrive, or whose own flag slot never rises."""
    from fp8gq import _lib, ops
    lib = _lib.load()
    dev = cuda_device
    stream = ops._stream(dev)
    pair = _Pair(dev)
    # one tagged call has happened on this rank (sequence 1) and only its own
    # half of the input words carries tag 1: rank 1's half is stale (tag 0)
    pair.state[1] = 1
    pair.flags[0][0] = 1
    xin = pair.words(M, K)
    g = torch.Generator(device=dev).manual_seed(M)
    xv = torch.randn(M, K, generator=g, device=dev).bfloat16()
    xin[0][:, :K // 4] = _tagged(xv[:, :K // 2], 1)
    xin[0][:, K // 4:] = _tagged(xv[:, K // 2:], 0)
    wq, ws = _weight(N, K, 7, dev)
    out = pair.words(M, 2 * N)
    nbytes = lib.fp8gq_workspace_bytes(M, N, K)
    work = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=dev)

    def consumer():
        return lib.fp8gq_fused_gemv_quant_gather(xin[0].data_ptr(), K, wq.data_ptr(), K, ws.data_ptr(), K // 128,
                                                 M, N, K, ctypes.byref(pair.desc(out, True)),
                                                 work.data_ptr() if nbytes else None, nbytes, stream)
    st, dt = _timed(consumer)
    _gave_up(fp8gq, lib, st, dt)

    # the decode kernel on the same stale words
    dst = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    pair.state[1] = 1
    st, dt = _timed(lambda: lib.fp8gq_gather_decode(ctypes.byref(pair.desc(xin, True)), M, K, dst.data_ptr(), K,
                                                    stream))
    _gave_up(fp8gq, lib, st, dt)

    # a publishing call without an input wait: rank 1's own flag slot is
    # behind this rank's sequence number (rank 1 never finished call 1)
    pair.state[1] = 1
    pair.flags[1][1] = 0
    xb = xv.contiguous()

    def publisher():
        return lib.fp8gq_fused_gemv_quant_gather(xb.data_ptr(), K, wq.data_ptr(), K, ws.data_ptr(), K // 128,
                                                 M, N, K, ctypes.byref(pair.desc(out, False)),
                                                 work.data_ptr() if nbytes else None, nbytes, stream)
    st, dt = _timed(publisher)
    _gave_up(fp8gq, lib, st, dt)

    # the context is usable: an ordinary call passes parity against the oracle
    o, xq, sx = fp8gq.fused_gemv_quant(xv, wq, ws, return_quant=True)
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    _, exact, rq, rs = O.fused_gemv_quant(to_f32(xv), to_u8(wq), to_f32(ws))
    assert (to_u8(xq) == rq).all() and (to_f32(sx) == rs).all()
    assert_close(to_f32(o), exact, 3.0)
