"""The N-sharded linear on CPU ranks (gloo, world size 2): every rank ends
with the full output, equal to the unsharded oracle.  The fused op is the
oracle here; the GPU path swaps in fp8gq.fused_gemv_quant and NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_op(x, Wq, Ws):
    from oracle import fp8gq_oracle as O
    from tests._util import bf16_tensor
    out, _, _, _ = O.fused_gemv_quant(x.float().numpy(), Wq.view(torch.uint8).numpy(), Ws.numpy())
    return bf16_tensor(out)


def _worker(rank, world, port, M, K, N, q):
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "sglang-triton-fusion_b200")]
    import torch.distributed as dist
    from oracle import fp8gq_oracle as O
    from tests._util import bf16_tensor, f32_tensor, fp8_tensor
    from fp8gq import dist as fd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = bf16_tensor(O.make_activation(M, K, seed=3))
        wq, ws = O.make_weight(N, K, seed=4)
        Wq, Ws = fp8_tensor(wq), f32_tensor(ws)
        w_r, s_r = fd.shard_rows(Wq, Ws, rank, world)
        out = fd.gathered_linear(x, w_r, s_r, op=_oracle_op)
        full = _oracle_op(x, Wq, Ws)
        q.put((rank, bool(torch.equal(out, full)), tuple(out.shape)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("M", [1, 3])
def test_sharded_linear_gloo_world2(M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, K, N = 2, 256, 512
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, M, K, N, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, equal, shape in res:
        assert equal, f"rank {rank}: gathered output differs from the unsharded oracle"
        assert shape == (M, N)


def test_shard_rows_rejects_uneven():
    from fp8gq import dist as fd
    from fp8gq.ops import ShapeError
    w = torch.zeros(384, 128, dtype=torch.float8_e4m3fn)
    s = torch.ones(3, 1)
    with pytest.raises(ShapeError):
        fd.shard_rows(w, s, 0, 2)
    a, b = fd.shard_rows(w, s, 1, 3)
    assert a.shape == (128, 128) and b.shape == (1, 1)
    assert np.shares_memory(a.view(torch.uint8).numpy(), w.view(torch.uint8).numpy())


def test_shard_cols_and_gate_up():
    from fp8gq import dist as fd
    from fp8gq.ops import ShapeError
    codes = torch.arange(256 * 512, dtype=torch.int32).remainder(120).to(torch.uint8).view(256, 512)
    w = codes.view(torch.float8_e4m3fn)
    s = torch.arange(2 * 4, dtype=torch.float32).view(2, 4)
    cols = [fd.shard_cols(w, s, r, 2) for r in range(2)]
    assert torch.equal(torch.cat([c[0].view(torch.uint8) for c in cols], 1), codes)
    assert torch.equal(torch.cat([c[1] for c in cols], 1), s)
    with pytest.raises(ShapeError):
        fd.shard_cols(w, s, 0, 3)
    # merged [gate; up] with I = 128: rank r gets gate rows [64r..] ... in 128-row blocks
    gw = codes[:, :128].contiguous().view(torch.float8_e4m3fn)      # [256, 128]: gate rows 0..127, up 128..255
    gs = torch.tensor([[1.0], [2.0]])
    gq, gss = fd.shard_gate_up(gw, gs, 0, 1)
    assert torch.equal(gq.view(torch.uint8), codes[:, :128]) and torch.equal(gss, gs)
    big = torch.arange(512 * 128, dtype=torch.int32).remainder(100).to(torch.uint8).view(512, 128)
    bs = torch.arange(4, dtype=torch.float32).view(4, 1)
    q1, s1 = fd.shard_gate_up(big.view(torch.float8_e4m3fn), bs, 1, 2)
    assert torch.equal(q1.view(torch.uint8), torch.cat([big[128:256], big[384:512]]))
    assert torch.equal(s1, torch.tensor([[1.0], [3.0]]))


def _paired_worker(rank, world, port, q):
    """One MLP block of paired tensor parallelism on CPU ranks with the
    oracle as the op: row-parallel partials, all-gathered (the GPU path stores
    them into every rank's slabs), summed in rank order by the reduce + norm
    prologue of the column-parallel gate_up, SwiGLU + down row-parallel, and the
    second reduce -- against the same block unsharded."""
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "sglang-triton-fusion_b200")]
    import torch.distributed as dist
    from oracle import fp8gq_oracle as O
    from tests._util import f32_tensor, fp8_tensor
    from fp8gq import dist as fd
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H, I = 512, 1024
        a = O.make_activation(1, H, seed=21)                    # the attention output (replicated stand-in)
        res0 = O.bf16_round(O.make_activation(1, H, seed=22, outlier_frac=0.0))
        nw = O.bf16_round((np.random.default_rng(23).standard_normal(H) * 0.1 + 1).astype(np.float32))
        wo, so = O.make_weight(H, H, seed=24)
        wgu, sgu = O.make_weight(2 * I, H, seed=25)
        wd, sd = O.make_weight(H, I, seed=26)

        def allgather(p):
            t = torch.from_numpy(np.ascontiguousarray(p, np.float32))
            outs = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(outs, t)
            return [o.numpy() for o in outs]

        # o_proj, row-parallel: this rank's K slice of the attention output
        Wo_r, So_r = fd.shard_cols(fp8_tensor(wo), f32_tensor(so), rank, world)
        kr = H // world
        po, _, _, _ = O.fused_gemv_quant(a[:, rank * kr:(rank + 1) * kr], Wo_r.view(torch.uint8).numpy(),
                                         So_r.numpy())
        parts_o = allgather(po)
        # gate_up, column-parallel (gate and up rows of this rank together)
        Wgu_r, Sgu_r = fd.shard_gate_up(fp8_tensor(wgu), f32_tensor(sgu), rank, world)
        gu_r, _, _, _, res1 = O.fused_reduce_add_rmsnorm_gemv_quant(parts_o, res0, nw, Wgu_r.view(torch.uint8).numpy(),
                                                                  Sgu_r.numpy())
        # down, row-parallel with the SwiGLU prologue on the local [gate | up]
        Wd_r, Sd_r = fd.shard_cols(fp8_tensor(wd), f32_tensor(sd), rank, world)
        pd, _, _, _ = O.fused_swiglu_q_gemm(gu_r, Wd_r.view(torch.uint8).numpy(), Sd_r.numpy())
        parts_d = allgather(pd)
        h2, res2, _ = O.reduce_add_rmsnorm(parts_d, res1, nw)
        # unsharded: o, add + norm, gate_up, SwiGLU + down, add + norm
        o_full, _, _, _ = O.fused_gemv_quant(a, wo, so)
        gu_full, _, _, _, r1f = O.fused_add_rmsnorm_gemv_quant(o_full, res0, nw, wgu, sgu)
        d_full, _, _, _ = O.fused_swiglu_q_gemm(gu_full, wd, sd)
        h2f, _, _ = O.add_rmsnorm(d_full, r1f, nw)
        q.put((rank, bool(O.rms_tolerance_ok(h2, h2f, rtol=5e-2, atol_rel_rms=5e-2)),
               float(np.abs(h2 - h2f).max()), bool(np.array_equal(res1, allgather(res1)[0]))))
    finally:
        dist.destroy_process_group()


def test_paired_mlp_block_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = _free_port()
    procs = [ctx.Process(target=_paired_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, maxdiff, same_res in res:
        assert ok, f"rank {rank}: paired block differs from the unsharded block (max |diff| {maxdiff})"
        assert same_res, f"rank {rank}: the residual differs between ranks"
