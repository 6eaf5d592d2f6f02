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
