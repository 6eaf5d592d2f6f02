"""Chain runner (fp8gq_chain_*) on one GPU.

A list of M == 1 linears runs as one cooperative launch; each linear polls the
tagged words of the earlier linear it reads.  The chain below has a skip
connection (a linear reading an output three links back), a SwiGLU link over
a [gate | up] output, a K = 12288 link (one weight row per ring stage, rows
taken in pairs) and a width that is not a power of two.  Every output must
equal, bit for bit, the row kernel on the same (decoded) input -- the chain
runs the row kernel's math in its order -- carry its link's sequence number,
and stay within the oracle's tolerance; a second launch must reproduce the
outputs with the sequence numbers moved on by the length of the list.  A chain
on a two-rank descriptor whose peer never writes gives up after the peer
limit, and the context stays usable.
"""
import ctypes
import time

import pytest
import torch

from oracle import fp8gq_oracle as O
from tests._util import assert_close, to_f32, to_u8

pytestmark = pytest.mark.gpu

LIMIT_NS = 200_000_000
SITE_GATHER = 0x80000000 | 8


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


# (K of the input it reads, N, src, swiglu): src -1 is the bf16 step input;
# a link reads the first K (2K with swiglu) columns of linear src's output
CHAIN = [
    (2048, 3072, -1, False),
    (1024, 2048, 0, False),      # first 1024 of 3072 columns
    (1024, 1024, 1, True),       # SwiGLU of [gate | up] = 2048 columns
    (3072, 1024, 0, False),      # skip connection: all of linear 0
    (1024, 12288, 3, False),
    (12288, 1024, 4, False),     # K = 12288: one row per stage, rows in pairs
    (1024, 1536, 5, False),
]


def _build(fp8gq, dev):
    g = torch.Generator(device=dev).manual_seed(9)
    x = torch.randn(1, CHAIN[0][0], generator=g, device=dev).bfloat16()
    links, weights, outs = [], [], []
    for i, (K, N, src, sw) in enumerate(CHAIN):
        wq, ws = _weight(N, K, 100 + i, dev)
        out = torch.zeros(1, N // 2, dtype=torch.int64, device=dev)
        xin = x if src < 0 else outs[src][:, :(2 * K if sw else K) // 2]
        links.append(fp8gq.Link(x=xin, w=wq, ws=ws, out=out, src=src, swiglu=sw))
        weights.append((wq, ws))
        outs.append(out)
    return x, links, weights, outs


def test_chain_matches_the_row_kernel(fp8gq, cuda_device):
    from fp8gq.dist import tags, untag
    dev = cuda_device
    torch.cuda.synchronize()
    fp8gq.device_error(clear=True)
    x, links, weights, outs = _build(fp8gq, dev)
    runner = fp8gq.ChainRunner(links)
    n = len(CHAIN)
    for launch in range(2):
        runner.run()
        torch.cuda.synchronize()
        assert fp8gq.device_error() == 0, hex(fp8gq.device_error())
        decoded = []
        for i, (K, N, src, sw) in enumerate(CHAIN):
            got = untag(outs[i])
            tg = tags(outs[i])
            assert bool((tg == launch * n + i + 1).all()), f"link {i}: tags {sorted(set(tg.flatten().tolist()))}"
            xin = x if src < 0 else decoded[src][:, :(2 * K if sw else K)].contiguous()
            wq, ws = weights[i]
            if sw:
                ref = fp8gq.fused_swiglu_q_gemm(xin, wq, ws)      # M == 1, 1 MB: the row kernel
                _, exact, _, _ = O.fused_swiglu_q_gemm(to_f32(xin), to_u8(wq), to_f32(ws))
            else:
                ref = fp8gq.fused_gemv_quant(xin, wq, ws, kernel="row")
                _, exact, _, _ = O.fused_gemv_quant(to_f32(xin), to_u8(wq), to_f32(ws))
            assert torch.equal(got, ref), f"link {i} (launch {launch}): differs from the row kernel in " \
                                          f"{(got != ref).sum().item()} of {N} columns"
            assert_close(to_f32(got), exact, 3.0)
            decoded.append(got)
        assert int(runner.state[1]) == (launch + 1) * n and int(runner.flags[0]) == (launch + 1) * n
        assert int(runner.state[0]) == 0
    # the decode kernel reads the last link's words
    y = runner.decode(outs[-1])
    torch.cuda.synchronize()
    assert torch.equal(y, untag(outs[-1]))
    assert fp8gq.device_error() == 0


def test_chain_argument_checks(fp8gq, cuda_device):
    from fp8gq import _lib
    dev = cuda_device
    x, links, _, outs = _build(fp8gq, dev)
    bad = list(links)
    bad[1] = fp8gq.Link(x=outs[2][:, :512], w=links[1].w, ws=links[1].ws, out=links[1].out, src=2)
    with pytest.raises(_lib.Fp8gqError):      # a link may read only an earlier link
        fp8gq.ChainRunner(bad)
    wq, ws = _weight(1024, 16384, 1, dev)
    big = [fp8gq.Link(x=torch.zeros(1, 16384, dtype=torch.bfloat16, device=dev), w=wq, ws=ws,
                      out=torch.zeros(1, 512, dtype=torch.int64, device=dev))]
    with pytest.raises(_lib.Fp8gqError):      # K above 12288
        fp8gq.ChainRunner(big)


@pytest.fixture
def short_limit(fp8gq):
    torch.cuda.synchronize()
    fp8gq.device_error(clear=True)
    prev = fp8gq.set_wait_limit_ns(LIMIT_NS)
    yield
    torch.cuda.synchronize()
    fp8gq.set_wait_limit_ns(prev)
    fp8gq.device_error(clear=True)


def test_chain_gives_up_on_a_silent_peer(fp8gq, cuda_device, short_limit):
    """A two-rank chain for rank 0 whose rank-1 buffers are local and never
    written: link 1 reads link 0's full output, whose rank-1 half never
    arrives."""
    from fp8gq import _lib, ops
    from fp8gq.dist import tags
    dev = cuda_device
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(1, 2048, generator=g, device=dev).bfloat16()
    flags = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(2)]
    state = torch.zeros(2, dtype=torch.int32, device=dev)
    w0, s0 = _weight(1024, 2048, 1, dev)          # rank 0's half of a 2048-row linear
    w1, s1 = _weight(1024, 2048, 2, dev)
    o0 = [torch.zeros(1, 1024, dtype=torch.int64, device=dev) for _ in range(2)]
    o1 = [torch.zeros(1, 1024, dtype=torch.int64, device=dev) for _ in range(2)]
    table = (_lib.ChainLinear * 2)()
    for i, (xp, w, s, out, src) in enumerate(((x.data_ptr(), w0, s0, o0, -1), (o0[0].data_ptr(), w1, s1, o1, 0))):
        t = table[i]
        t.x, t.w, t.ldw, t.ws, t.ldws = xp, w.data_ptr(), 2048, s.data_ptr(), 16
        t.N, t.K, t.src, t.swiglu, t.col0, t.reserved = 1024, 2048, src, 0, 0, 0
        for r in range(2):
            t.out[r] = out[r].data_ptr()
    gd = _lib.Gather()
    for q in range(2):
        gd.flags[q] = flags[q].data_ptr()
    gd.counter, gd.seq = state.data_ptr(), state.data_ptr() + 4
    gd.world, gd.rank, gd.tagged = 2, 0, 1
    nbytes = lib.fp8gq_chain_plan_bytes(2)
    mem = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
    plan = _lib.ChainPlan()
    st = lib.fp8gq_chain_prepare(table, 2, ctypes.byref(gd), (mem.data_ptr() + 255) // 256 * 256, nbytes,
                                 ctypes.byref(plan))
    assert st == 0, lib.fp8gq_status_string(st)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = lib.fp8gq_chain_run(ctypes.byref(plan), ops._stream(dev))
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert st == 0, lib.fp8gq_status_string(st)
    assert 0.8 * LIMIT_NS * 1e-9 <= dt < 2.0 * LIMIT_NS * 1e-9 + 0.5, f"chain took {dt:.3f} s"
    assert fp8gq.device_error() == SITE_GATHER, hex(fp8gq.device_error())
    fp8gq.device_error(clear=True)
    # link 0 (bf16 input) was not held up: its half carries tag 1 on both buffers
    assert bool((tags(o0[0][:, :512]) == 1).all()) and torch.equal(o0[0][:, :512], o0[1][:, :512])
    # the context is usable
    o, xq, sx = fp8gq.fused_gemv_quant(x, w0, s0, return_quant=True)
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    _, exact, rq, rs = O.fused_gemv_quant(to_f32(x), to_u8(w0), to_f32(s0))
    assert (to_u8(xq) == rq).all()
    assert_close(to_f32(o), exact, 3.0)
