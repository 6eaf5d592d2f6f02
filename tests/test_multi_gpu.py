"""N-sharded linears on 2, 4 and 8 GPUs (one process per GPU, NCCL process
group), each world size skipped where the box has fewer GPUs.

The op being sharded is fused_gemv_quant (kernels/fused_gemv_quant_tm.py:83-102):
rank r holds rows [r*N/w, (r+1)*N/w) of every weight, and the kernels store
their output slices into every rank's buffer over NVLink (fp8gq.dist.PeerGather).

* A chain of gathered linears whose outputs ping-pong between two buffers --
  each linear reads the previous one's gathered output and overwrites the
  buffer its predecessor read -- with the ranks pushed out of step by sleep
  kernels.  Every stage's full output, on every rank, must be bit-identical
  across ranks and within the tile kernel's tolerance of the oracle of the
  *unsharded* linear; a second run of the chain, twice back to back with no
  wait between, must reproduce the final output bit for bit (a store that
  overtook a slower rank still reading its buffer would change it).
* The NCCL all-gather baseline against the same oracle.
* Paired tensor parallelism: row-parallel partials stored into every rank's
  slab, summed by the next column-parallel linear's reduce + add + RMSNorm
  prologue; each stage against the oracle.
* The M = 1 tagged chain as one persistent launch (fp8gq.ChainRunner): every
  stage against the oracle and across ranks, reruns with a rank held back.
* The same chains with tagged words (PeerGather(tagged=True)): each linear
  reads the previous one's tagged output directly, the last stage of each
  chain a SwiGLU over a gathered [gate | up] output; every stage decoded on
  every rank against the oracle and across ranks, the back-to-back reruns
  with one rank held back, and every word of the final output carrying the
  sequence number of the call that wrote it.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLDS = [2, 4, 8]

# chains (M, widths): linear j maps widths[j] -> widths[j + 1]; every width is
# a multiple of 1024 so that 128-row blocks split evenly over 8 ranks.  At
# M = 1 the unsharded weights span both kernels (row <= 20 MiB < tile) and a
# long-K linear (12288 -> 4096); M = 4 runs the tile kernel.
CHAINS = [(1, [4096, 6144, 4096, 4096, 12288, 4096, 4096]), (4, [2048, 3072, 2048, 2048])]
SKEW_CYCLES = 400_000      # ~0.2 ms sleep kernel that pushes one rank behind
# tagged chains (M, stages): stage (K, N, swiglu) maps an input of K columns
# (2K for a SwiGLU stage, which reads the previous [gate | up] output) to N.
# At M = 1 the shards span the row kernel (one, two and four rows per group)
# and the tile kernel; M = 4 runs the tile kernel.
TAGGED_CHAINS = [(1, [(4096, 6144, False), (6144, 4096, False), (4096, 12288, False), (12288, 4096, False),
                      (4096, 6144, False), (3072, 4096, True)]),
                 (4, [(2048, 3072, False), (3072, 2048, False), (2048, 2048, False), (1024, 2048, True)])]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weight(N, K, seed, dev):
    """The full (unsharded) e4m3 weight and block scales; every rank makes the
    same one from the seed and takes its slice."""
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = (blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0).contiguous()
    return (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K).contiguous(), ws


def _activation(M, K, seed, dev, std=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=dev) * std
    ch = torch.randperm(K, generator=g, device=dev)[: max(1, K // 100)]
    x[:, ch] *= 20.0
    return x.bfloat16()


def _setup(rank, world, port):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "sglang-triton-fusion_b200")]
    from datetime import timedelta

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=120))
    return dev


def _oracle_check(errs, what, got, x, wq, ws, ulps=3.0, swiglu=False):
    """got (full output) within the ulp tolerance of the oracle of the
    unsharded linear on input x."""
    from oracle import fp8gq_oracle as O
    from tests._util import to_f32, to_u8
    fn = O.fused_swiglu_q_gemm if swiglu else O.fused_gemv_quant
    _, exact, _, _ = fn(to_f32(x), to_u8(wq), to_f32(ws))
    g = to_f32(got).astype(np.float64)
    atol = O.ref_atol(exact, ulps)
    if not (O.rms_tolerance_ok(g, exact) and np.all(np.abs(g - exact) <= atol)):
        d = np.abs(g - exact).max()
        errs.append(f"{what}: max |err| {d:.4g} > {ulps} ulp ({atol:.4g}) of the oracle")


def _same_on_every_rank(errs, what, t):
    """t bit-identical to rank 0's copy."""
    import torch.distributed as dist
    ref = t.clone()
    dist.broadcast(ref, src=0)
    if not torch.equal(ref, t):
        errs.append(f"{what}: differs from rank 0's copy in {(ref != t).sum().item()} elements")


def _chain_worker(rank, world, port, result_q):
    dev = _setup(rank, world, port)
    import torch.distributed as dist

    import fp8gq
    from fp8gq import dist as fdist
    errs = []
    try:
        fp8gq.load()
        for ci, (M, widths) in enumerate(CHAINS):
            n = len(widths) - 1
            wmax = max(widths[1:])
            buf = torch.zeros(2 * M * wmax + 64, dtype=torch.bfloat16, device=dev)
            pg = fdist.PeerGather(buf)
            bufs = [buf[:M * wmax], buf[M * wmax:2 * M * wmax]]
            lins = []
            for j in range(n):
                K, N = widths[j], widths[j + 1]
                wq, ws = _weight(N, K, 1000 * ci + j, dev)
                lins.append((wq, ws) + fdist.shard_rows(wq, ws, rank, world))
            x0 = _activation(M, widths[0], 77 + ci, dev)

            def out_of(j):
                return bufs[j % 2].view(-1)[:M * widths[j + 1]].view(M, widths[j + 1])

            def run(snapshots=None, skew_at=None):
                for j in range(n):
                    if skew_at is not None and rank == skew_at(j):
                        torch.cuda._sleep(SKEW_CYCLES)
                    x = x0 if j == 0 else out_of(j - 1)
                    pg.linear(x, lins[j][2], lins[j][3], out_of(j), wait_input=j > 0)
                    if snapshots is not None:
                        pg.wait(out_of(j))
                        snapshots.append(out_of(j).clone())

            # pass 1: a snapshot of every stage (each after a wait for all slices)
            snaps = []
            run(snaps, skew_at=lambda j: j % world)
            torch.cuda.synchronize()
            for j in range(n):
                _same_on_every_rank(errs, f"chain {ci} M={M} stage {j}", snaps[j])
            if rank == 0:
                for j in range(n):
                    x = x0 if j == 0 else snaps[j - 1]
                    _oracle_check(errs, f"chain {ci} M={M} stage {j} ({widths[j]}->{widths[j + 1]})",
                                  snaps[j], x, lins[j][0], lins[j][1])
            # pass 2: the chain twice back to back, nothing in between; the
            # last rank falls behind right before each pass's last linear, so
            # the next pass's first linear (which does not wait for an input)
            # is ready to store into buffers that rank is still reading
            dist.barrier()
            run(skew_at=lambda j: world - 1 if j == n - 1 else None)
            run(skew_at=lambda j: world - 1 if j == n - 1 else None)
            pg.wait(out_of(n - 1))
            torch.cuda.synchronize()
            if not torch.equal(out_of(n - 1), snaps[n - 1]):
                errs.append(f"chain {ci} M={M}: back-to-back rerun changed the final output in "
                            f"{(out_of(n - 1) != snaps[n - 1]).sum().item()} elements")
            # NCCL all-gather baseline on the same stage inputs
            for j in range(n):
                x = x0 if j == 0 else snaps[j - 1]
                full = fdist.gathered_linear(x, lins[j][2], lins[j][3])
                if rank == 0:
                    _oracle_check(errs, f"chain {ci} M={M} stage {j} via NCCL", full, x, lins[j][0], lins[j][1])
            if fp8gq.device_error() != 0:
                errs.append(f"device error word {fp8gq.device_error():#x}")
            pg.close()
        result_q.put((rank, errs))
    except Exception as e:          # report instead of leaving the other ranks waiting
        result_q.put((rank, errs + [f"exception: {e!r}"]))
        raise
    finally:
        dist.destroy_process_group()


def _spawn(target, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, errs = q.get(timeout=600)
            results[rank] = errs
    finally:
        for p in procs:
            p.join(timeout=180)
            if p.exitcode is None:
                p.kill()
    for rank, errs in sorted(results.items()):
        assert not errs, f"rank {rank}: {errs}"
    for p in procs:
        assert p.exitcode == 0


def _skip_unless(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")


@pytest.mark.parametrize("world", WORLDS)
def test_gathered_chain_matches_oracle(world):
    _skip_unless(world)
    _spawn(_chain_worker, world)


def _tagged_chain_worker(rank, world, port, result_q):
    dev = _setup(rank, world, port)
    import torch.distributed as dist

    import fp8gq
    from fp8gq import dist as fdist
    errs = []
    try:
        fp8gq.load()
        for ci, (M, stages) in enumerate(TAGGED_CHAINS):
            n = len(stages)
            wmax = max(N for _, N, _ in stages)
            words = torch.zeros(M * wmax + 32, dtype=torch.int64, device=dev)   # two buffers of M * wmax / 2
            pg = fdist.PeerGather(words, tagged=True)
            bufs = [words[:M * wmax // 2], words[M * wmax // 2:M * wmax]]
            lins = []
            for j, (K, N, sw) in enumerate(stages):
                wq, ws = _weight(N, K, 5000 + 100 * ci + j, dev)
                lins.append((wq, ws) + fdist.shard_rows(wq, ws, rank, world))
            x0 = _activation(M, stages[0][0], 91 + ci, dev)

            def out_of(j):
                N = stages[j][1]
                return bufs[j % 2].view(-1)[:M * N // 2].view(M, N // 2)

            def run(snapshots=None, skew_at=None):
                for j, (K, N, sw) in enumerate(stages):
                    if skew_at is not None and rank == skew_at(j):
                        torch.cuda._sleep(SKEW_CYCLES)
                    x = x0 if j == 0 else out_of(j - 1)
                    call = pg.swiglu_linear if sw else pg.linear
                    call(x, lins[j][2], lins[j][3], out_of(j), wait_input=j > 0)
                    if snapshots is not None:
                        snapshots.append(pg.decode(out_of(j)))

            snaps = []
            run(snaps, skew_at=lambda j: j % world)
            torch.cuda.synchronize()
            for j in range(n):
                _same_on_every_rank(errs, f"tagged chain {ci} M={M} stage {j}", snaps[j])
            if rank == 0:
                for j, (K, N, sw) in enumerate(stages):
                    x = x0 if j == 0 else snaps[j - 1]
                    _oracle_check(errs, f"tagged chain {ci} M={M} stage {j} ({'swiglu ' if sw else ''}{K}->{N})",
                                  snaps[j], x, lins[j][0], lins[j][1], swiglu=sw)
            dist.barrier()
            run(skew_at=lambda j: world - 1 if j == n - 1 else None)
            run(skew_at=lambda j: world - 1 if j == n - 1 else None)
            final = pg.decode(out_of(n - 1))
            torch.cuda.synchronize()
            if not torch.equal(final, snaps[n - 1]):
                errs.append(f"tagged chain {ci} M={M}: back-to-back rerun changed the final output in "
                            f"{(final != snaps[n - 1]).sum().item()} elements")
            tg = fdist.tags(out_of(n - 1))
            if not bool((tg == 3 * n).all()):
                errs.append(f"tagged chain {ci} M={M}: final words tagged {sorted(set(tg.flatten().tolist()))}, "
                            f"expected {3 * n}")
            if fp8gq.device_error() != 0:
                errs.append(f"device error word {fp8gq.device_error():#x}")
            pg.close()
        result_q.put((rank, errs))
    except Exception as e:
        result_q.put((rank, errs + [f"exception: {e!r}"]))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_tagged_chain_matches_oracle(world):
    _skip_unless(world)
    _spawn(_tagged_chain_worker, world)


def _chain_runner_worker(rank, world, port, result_q):
    """The M = 1 tagged chain as one persistent launch (fp8gq.ChainRunner),
    every stage in its own buffer so that each can be checked afterwards."""
    dev = _setup(rank, world, port)
    import torch.distributed as dist

    import fp8gq
    from fp8gq import dist as fdist
    errs = []
    try:
        fp8gq.load()
        for ci, (M, stages) in enumerate(TAGGED_CHAINS):
            if M != 1:
                continue
            n = len(stages)
            sizes = [N // 2 for _, N, _ in stages]
            words = torch.zeros(sum(sizes) + 32, dtype=torch.int64, device=dev)
            pg = fdist.PeerGather(words, tagged=True)
            outs, off = [], 0
            for sz in sizes:
                outs.append(words[off:off + sz].view(1, sz))
                off += sz
            lins, links = [], []
            x0 = _activation(1, stages[0][0], 191 + ci, dev)
            for j, (K, N, sw) in enumerate(stages):
                wq, ws = _weight(N, K, 7000 + 100 * ci + j, dev)
                lins.append((wq, ws) + fdist.shard_rows(wq, ws, rank, world))
                x = x0 if j == 0 else outs[j - 1][:, :(2 * K if sw else K) // 2]
                links.append(fp8gq.Link(x=x, w=lins[j][2], ws=lins[j][3], out=outs[j], src=j - 1, swiglu=sw))
            runner = fp8gq.ChainRunner(links, gather=pg)
            runner.run()
            final = runner.decode(outs[-1])
            torch.cuda.synchronize()
            dist.barrier()
            snaps = [fdist.untag(o) for o in outs[:-1]] + [final]
            for j in range(n):
                _same_on_every_rank(errs, f"chain runner {ci} stage {j}", snaps[j])
            if rank == 0:
                for j, (K, N, sw) in enumerate(stages):
                    x = x0 if j == 0 else snaps[j - 1][:, :2 * K if sw else K]
                    _oracle_check(errs, f"chain runner {ci} stage {j} ({'swiglu ' if sw else ''}{K}->{N})",
                                  snaps[j], x, lins[j][0], lins[j][1], swiglu=sw)
            # twice more back to back, the last rank held back before each
            dist.barrier()
            for _ in range(2):
                if rank == world - 1:
                    torch.cuda._sleep(SKEW_CYCLES)
                runner.run()
            again = runner.decode(outs[-1])
            torch.cuda.synchronize()
            if not torch.equal(again, final):
                errs.append(f"chain runner {ci}: rerun changed the final output in "
                            f"{(again != final).sum().item()} elements")
            for j in range(n):
                tg = fdist.tags(outs[j])
                if not bool((tg == 2 * n + j + 1).all()):
                    errs.append(f"chain runner {ci} stage {j}: tags {sorted(set(tg.flatten().tolist()))[:4]}, "
                                f"expected {2 * n + j + 1}")
            if fp8gq.device_error() != 0:
                errs.append(f"device error word {fp8gq.device_error():#x}")
            dist.barrier()
            pg.close()
        result_q.put((rank, errs))
    except Exception as e:
        result_q.put((rank, errs + [f"exception: {e!r}"]))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_chain_runner_matches_oracle(world):
    _skip_unless(world)
    _spawn(_chain_runner_worker, world)


def _paired_worker(rank, world, port, result_q):
    """One attention-to-MLP block of paired tensor parallelism: row-parallel
    o_proj stores its partial into every rank's slab, column-parallel gate_up
    sums the slabs in its reduce + add + RMSNorm prologue, the SwiGLU +
    down_proj partials go to the second set of slabs, and a second reduce +
    norm linear (the next layer's qkv) sums them.  Each rank checks its own
    stages against the oracle; the slabs must be identical on every rank."""
    dev = _setup(rank, world, port)
    import torch.distributed as dist

    import fp8gq
    from fp8gq import dist as fdist
    from oracle import fp8gq_oracle as O
    from tests._util import to_f32, to_u8
    errs = []
    try:
        fp8gq.load()
        H, I, NQ = 4096, 6144, 6144
        for M in (1, 4):
            buf = torch.zeros(2 * world * M * H + 64, dtype=torch.bfloat16, device=dev)
            pg = fdist.PeerGather(buf)
            slabs_o = buf[:world * M * H].view(world, M, H)
            slabs_d = buf[world * M * H:2 * world * M * H].view(world, M, H)
            a = _activation(M, H, 40 + M, dev)
            g = torch.Generator(device=dev).manual_seed(50 + M)
            res0 = torch.randn(M, H, generator=g, device=dev).bfloat16()
            nw = (torch.randn(H, generator=g, device=dev) * 0.1 + 1).bfloat16()
            wo, so = _weight(H, H, 41, dev)
            wgu, sgu = _weight(2 * I, H, 42, dev)
            wd, sd = _weight(H, I, 43, dev)
            wq, sq = _weight(NQ, H, 44, dev)
            kr = H // world
            wo_r, so_r = fdist.shard_cols(wo, so, rank, world)
            wgu_r, sgu_r = fdist.shard_gate_up(wgu, sgu, rank, world)
            wd_r, sd_r = fdist.shard_cols(wd, sd, rank, world)
            wq_r, sq_r = fdist.shard_rows(wq, sq, rank, world)
            a_r = a[:, rank * kr:(rank + 1) * kr]
            gu_r = torch.empty(M, wgu_r.shape[0], dtype=torch.bfloat16, device=dev)
            res1 = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            q_r = torch.empty(M, wq_r.shape[0], dtype=torch.bfloat16, device=dev)
            res2 = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
            pg.linear_partial(a_r, wo_r, so_r, slabs_o)
            pg.reduce_norm_linear(slabs_o, res0, nw, wgu_r, sgu_r, gu_r, res1)
            pg.linear_partial(gu_r, wd_r, sd_r, slabs_d, swiglu=True)
            pg.reduce_norm_linear(slabs_d, res1, nw, wq_r, sq_r, q_r, res2)
            pg.wait(slabs_d[rank])
            torch.cuda.synchronize()
            _same_on_every_rank(errs, f"M={M}: o partial slabs", slabs_o)
            _same_on_every_rank(errs, f"M={M}: down partial slabs", slabs_d)
            _same_on_every_rank(errs, f"M={M}: residual 1", res1)
            _same_on_every_rank(errs, f"M={M}: residual 2", res2)
            # this rank's row-parallel partials: the oracle of its K slice
            _oracle_check(errs, f"M={M}: o partial of rank {rank}", slabs_o[rank], a_r, wo_r, so_r)
            _oracle_check(errs, f"M={M}: down partial of rank {rank}", slabs_d[rank], gu_r, wd_r, sd_r,
                          swiglu=True)
            # the column-parallel linears: the sum of the landed slabs in rank
            # order + residual, norm, quant and GEMV of this rank's rows; the
            # new residual bit-exact
            for what, slabs, res_in, w_r, s_r, out, res_out in (
                    ("gate_up", slabs_o, res0, wgu_r, sgu_r, gu_r, res1),
                    ("qkv", slabs_d, res1, wq_r, sq_r, q_r, res2)):
                _, exact, _, _, res_o = O.fused_reduce_add_rmsnorm_gemv_quant(
                    [to_f32(slabs[q]) for q in range(world)], to_f32(res_in), to_f32(nw), to_u8(w_r),
                    to_f32(s_r))
                got = to_f32(out).astype(np.float64)
                atol = O.ref_atol(exact, 3.0)
                if not (O.rms_tolerance_ok(got, exact) and np.all(np.abs(got - exact) <= atol)):
                    errs.append(f"M={M}: {what} slice of rank {rank} outside 3 ulp of the oracle")
                if not np.array_equal(to_f32(res_out), res_o):
                    errs.append(f"M={M}: {what} residual_out != oracle (sum of slabs in rank order + residual)")
            if fp8gq.device_error() != 0:
                errs.append(f"device error word {fp8gq.device_error():#x}")
            pg.close()
        result_q.put((rank, errs))
    except Exception as e:
        result_q.put((rank, errs + [f"exception: {e!r}"]))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_paired_tensor_parallel_block_matches_oracle(world):
    _skip_unless(world)
    _spawn(_paired_worker, world)
