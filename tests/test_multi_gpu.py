"""N-sharded linears on two GPUs (one process per GPU, NCCL process group):
the output gathered by the kernels themselves over peer memory
(fp8gq.dist.PeerGather) and by an NCCL all-gather after the op, both against
the unsharded op on one GPU.  Skipped on boxes with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# (M, K, N): row kernel (M == 1, small weight), tile kernel at M == 1 and M == 4
CASES = [(1, 4096, 4096), (1, 4096, 24576), (4, 2048, 2560), (1, 12288, 4096)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weight(N, K, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = (blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0).contiguous()
    return (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K).contiguous(), ws


def _worker(rank, world, port, result_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "sglang-triton-fusion_b200")]
    from datetime import timedelta

    import torch.distributed as dist

    import fp8gq
    from fp8gq import dist as fdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        fp8gq.load()
        total = sum(M * N for M, _, N in CASES)
        buf = torch.zeros(total + 4096, dtype=torch.bfloat16, device=dev)
        pg = fdist.PeerGather(buf, group=None)
        errs = []
        outs, refs, nccl = [], [], []
        off = 0
        for i, (M, K, N) in enumerate(CASES):
            wq, ws = _weight(N, K, 10 + i, dev)
            gx = torch.Generator(device=dev).manual_seed(20 + i)
            x = torch.randn(M, K, generator=gx, device=dev).bfloat16()
            wq_r, ws_r = fdist.shard_rows(wq, ws, rank, world)
            out = buf[off:off + M * N].view(M, N)
            off += M * N
            pg.linear(x, wq_r, ws_r, out, wait_input=True)        # waits for the previous case's slices
            outs.append(out)
            refs.append(fp8gq.fused_gemv_quant(x, wq_r, ws_r))      # this rank's slice, unsharded op
            nccl.append(fdist.gathered_linear(x, wq_r, ws_r))
        pg.wait(outs[-1])
        torch.cuda.synchronize()
        # every rank's slice: gather the per-rank references with NCCL
        for i, (M, K, N) in enumerate(CASES):
            full = fdist.all_gather_columns(refs[i])
            if not torch.equal(outs[i], full):
                errs.append(f"case {i} p2p != per-rank op: {(outs[i] != full).sum().item()} elements")
            if not torch.equal(nccl[i], full):
                errs.append(f"case {i} nccl != per-rank op")
        if fp8gq.device_error() != 0:
            errs.append(f"device error word {fp8gq.device_error():#x}")
        pg.close()
        result_q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_gather_matches_per_rank_ops():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world = 2
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, errs = q.get(timeout=300)
        results[rank] = errs
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, errs in results.items():
        assert not errs, f"rank {rank}: {errs}"
