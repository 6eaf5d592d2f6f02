"""N-sharding of a block-FP8 linear across ranks (one process per GPU).

The output columns of a linear are independent, so rank r of `world` holds
rows [r*N/world, (r+1)*N/world) of the weight (whole 128-row blocks, so the
block scales split with it), runs the fused op on that slice and the bf16
slices are all-gathered (NCCL on GPUs).  The activation is replicated;
every rank quantises it itself.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import ops


def shard_rows(Wq: torch.Tensor, Ws: torch.Tensor, rank: int, world: int):
    """Rank `rank`'s slice of a weight [N, K] and its block scales [N/128, K/128]."""
    N = Wq.shape[0]
    nb = N // ops.GROUP
    if N % ops.GROUP or nb % world:
        raise ops.ShapeError(f"N/128 = {nb} row blocks do not split evenly over {world} ranks")
    per = nb // world
    return (Wq[rank * per * ops.GROUP:(rank + 1) * per * ops.GROUP],
            Ws[rank * per:(rank + 1) * per])


def all_gather_columns(shard: torch.Tensor, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """[M, Nr] per rank -> [M, world * Nr] with rank r's columns at r * Nr."""
    world = dist.get_world_size(group)
    M, Nr = shard.shape
    shard = shard.contiguous()
    gathered = torch.empty(world, M, Nr, dtype=shard.dtype, device=shard.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered.view(-1), shard.view(-1), group=group)
    else:
        dist.all_gather(list(gathered.unbind(0)), shard, group=group)
    if M == 1 and out is None:
        return gathered.view(1, world * Nr)
    res = gathered.permute(1, 0, 2).reshape(M, world * Nr)
    if out is not None:
        out.copy_(res)
        return out
    return res


def gathered_linear(x: torch.Tensor, Wq_shard: torch.Tensor, Ws_shard: torch.Tensor, group=None,
                    op=None) -> torch.Tensor:
    """fused_gemv_quant on this rank's rows, then the all-gather: the full
    (M, N) output on every rank.  `op` defaults to fp8gq.fused_gemv_quant."""
    op = op or ops.fused_gemv_quant
    return all_gather_columns(op(x, Wq_shard, Ws_shard), group=group)
