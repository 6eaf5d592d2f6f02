#!/usr/bin/env python
"""Benchmark of the fused FP8 quant + GEMV decode path on B200.

Workload (one "step" = one decode step's linear stack at M = 1): the Qwen3-8B
FP8 decoder's four block-FP8 linears -- qkv 4096->6144, o 4096->4096,
gate_up 4096->24576, down 12288->4096 -- for each of 36 layers, every layer
with its own seeded random e4m3 weights and 128x128 fp32 block scales
(W ~ N(0, 0.02^2) block-quantised, activations bf16 ~ N(0, 1) with 1% of the
channels x20).  6.95 GB of weights per step, far larger than the 126 MB L2,
so no L2 flush is needed between steps.  The weights are declared static
(fp8gq.set_static_weights; --static-weights 0 turns it off): nothing in a
decode step writes them, so each kernel may fetch its first weight tiles
before the previous kernel in the stream has finished.  With --gpus N > 1 the weights are
sharded across the ranks, so the total work is fixed (strong scaling):
--tp-mode paired makes qkv and gate_up column-parallel and o and
down row-parallel, the row-parallel kernels storing their partial outputs
into every rank's slabs over NVLink and the next column-parallel kernel
adding them in its add + RMSNorm prologue (two exchanges per layer);
--tp-mode tagged (default) shards every linear by output rows, its kernel
storing its slice into every rank's output as tagged words (bf16 pairs with
the call's sequence number) and each linear reading the previous one's output
-- qkv -> o -> gate_up -> down -> the next layer's qkv -- by polling the words
it reads; --tp-mode gather does the same with a flag raised after each
kernel's stores, every linear reading its own input; --tp-mode nccl shards
the same way and all-gathers with NCCL after each linear.

value     algorithmic bytes per step / device time per step (CUDA graph of one
          step, CUDA events, max over ranks), in GB/s (whole job).
e2e       the same metric through the public API (prepared launches of the
          fp8gq calls, each half of the step captured once into a CUDA graph
          and replayed, as a serving loop replays its decode step) with the
          step's inputs copied in from pinned host memory and its outputs
          copied back every step, inside the timed region (two copies of the
          buffers, so a step's copies overlap its neighbours' compute).
roofline  the dominant kernel (gate_up; at M = 1 the tile kernel): algorithmic
          bytes per launch / average launch duration (CUDA graph of 36 launches
          on distinct weights), against MEASURED_PEAKS.json's hbm_gbs.
cpu_baseline  the reference's PyTorch path (quantise, dequantise, fp32 matmul)
          on the host cores, on a bounded sample (rank 0, N = 1 only).

--impl reference runs that CPU reference path alone (rank 0; the other ranks
exit), one linear of the stack per step in rotation.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "sglang-triton-fusion_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

LAYERS = 36
SHAPES = [("qkv", 4096, 6144), ("o", 4096, 4096), ("gate_up", 4096, 24576), ("down", 12288, 4096)]
METRIC = "fused FP8 quant+GEMV achieved HBM GB/s, M=1, Qwen3-8B decode linear stack (36 layers)"
WORKLOAD = ("qwen3-8b-fp8 decode linear stack, M=1: 36 layers x {qkv 4096->6144, o 4096->4096, "
            "gate_up 4096->24576, down 12288->4096}, e4m3 weights with 128x128 fp32 block scales, "
            "bf16 activations with 1x128 group quant")


# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel,
# from the ncu captures summarised in profiles/ (single-GPU gate_up case)
NCU_TRAFFIC_BYTES = {"gemv_row_kernel<false>": 100_719_872 + 3_674_368,
                     "gemm_tm_kernel<16,false>": 100_815_616 + 3_400_448}   # keyed by ROUTED_KERNEL

# M == 1 routing of fp8gq_fused_gemv_quant / fp8gq_fused_swiglu_q_gemm: the row
# kernel for weights of at most 20 MiB (and K <= 49152), the tile kernel above.
ROW_PREFER_BYTES = 20 << 20


def ROUTED_KERNEL(N: int, K: int, swiglu: bool = False) -> str:
    sw = "true" if swiglu else "false"
    if N * K <= ROW_PREFER_BYTES and K <= 49152:
        return f"gemv_row_kernel<{sw}>"
    return f"gemm_tm_kernel<16,{sw}>"


def alg_bytes(M: int, K: int, N: int) -> int:
    """N*K weight bytes + fp32 block scales + bf16 activation in + bf16 out."""
    return N * K + 4 * (N // 128) * (K // 128) + 2 * M * K + 2 * M * N


STEP_BYTES = LAYERS * sum(alg_bytes(1, K, N) for _, K, N in SHAPES)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--e2e-steps", type=int, default=100)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--static-weights", type=int, default=1,
                    help="1 (default): declare the weights static (fp8gq.set_static_weights) -- no work "
                         "queued before a linear writes its weights, as in any decode step -- letting each "
                         "kernel fetch its first weight tiles before the previous one finishes; 0: do not")
    ap.add_argument("--tp-mode", choices=["paired", "gather", "tagged", "chain", "nccl"], default="tagged",
                    help="N > 1: paired -- qkv and gate_up column-parallel, o and down "
                         "row-parallel; each row-parallel kernel stores its partial into every rank's "
                         "slab over NVLink and the next column-parallel kernel adds the slabs in its "
                         "add + RMSNorm prologue (two exchanges per layer); gather -- every "
                         "linear N-sharded, the kernels store their output slices into every rank's buffer "
                         "and raise a flag; tagged (default) -- the same stores as tagged words, each linear "
                         "reading the previous one's output (qkv -> o -> gate_up -> down -> next qkv) and "
                         "polling the words it reads, no flags; chain -- the tagged step's 144 linears in "
                         "one persistent launch (fp8gq.ChainRunner); nccl -- every linear N-sharded, an NCCL "
                         "all-gather after each")
    ap.add_argument("--profile-case", default=None,
                    help="launch one kernel case --warmup + --steps times and exit (for ncu): "
                         "<shape>[:row|:tm][:M=<m>] with shape in qkv,o,gate_up,down,swiglu_down, "
                         "norm_<shape> (add + RMSNorm prologue), writer, add_rmsnorm, group_quant "
                         "(activation kernels alone, M rows), 'stack' for the whole decode step's "
                         "routed linears, or 'stack_runner[:L=<layers>]' for the decode chain in one "
                         "persistent launch")
    return ap.parse_args()


def measured_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------- NVLink --
class NvlinkCounter:
    """This GPU's NVLink traffic over a window, from the GPU performance
    monitor (NVML GPM samples before and after; read-only, nothing on the GPU
    is changed): total transmitted and received bytes per second over all
    links, times the window.  `error` holds the reason when the counters are
    not available (no GPM support, no pynvml)."""

    def __init__(self, dev_index: int):
        self.error = None
        self.nv = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            self.h = nv.nvmlDeviceGetHandleByIndex(dev_index)
            sup = nv.nvmlGpmQueryDeviceSupport(self.h)
            if not sup.isSupportedDevice:
                self.error = "GPM not supported on this device"
            else:
                self.s = [nv.nvmlGpmSampleAlloc(), nv.nvmlGpmSampleAlloc()]
        except Exception as e:          # counters are optional evidence
            self.error = f"{type(e).__name__}: {e}"

    def start(self):
        if self.error is None:
            try:
                self.nv.nvmlGpmSampleGet(self.h, self.s[0])
                self.t0 = time.monotonic()
            except Exception as e:
                self.error = f"{type(e).__name__}: {e}"

    def stop(self):
        """(tx bytes, rx bytes) over the window, or None."""
        if self.error is not None:
            return None
        try:
            nv = self.nv
            nv.nvmlGpmSampleGet(self.h, self.s[1])
            dt = time.monotonic() - self.t0
            mg = nv.c_nvmlGpmMetricsGet_t()
            mg.version = nv.NVML_GPM_METRICS_GET_VERSION
            mg.numMetrics = 2
            mg.sample1 = self.s[0]
            mg.sample2 = self.s[1]
            mg.metrics[0].metricId = nv.NVML_GPM_METRIC_NVLINK_TOTAL_TX_PER_SEC
            mg.metrics[1].metricId = nv.NVML_GPM_METRIC_NVLINK_TOTAL_RX_PER_SEC
            nv.nvmlGpmMetricsGet(mg)
            # the GPM rates are in MiB/s
            return (mg.metrics[0].value * 2**20 * dt, mg.metrics[1].value * 2**20 * dt, dt)
        except Exception as e:
            self.error = f"{type(e).__name__}: {e}"
            return None

    def close(self):
        if self.nv is not None:
            try:
                for smp in getattr(self, "s", []):
                    self.nv.nvmlGpmSampleFree(smp)
                self.nv.nvmlShutdown()
            except Exception:
                pass


# ------------------------------------------------------------- clocks --
class ClockSampler:
    """nvidia-smi samples of the job's GPUs (every rank's, identified by UUID),
    taken by one process on rank 0 while the GPUs run the step.  The timed
    region of a short run lasts milliseconds, less than the sampling period,
    so the bench keeps replaying the same step for a load window around it
    (untimed replays before and after) and the sampler covers that window;
    __enter__ returns once the first sample has arrived."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuids, active: bool = True):
        self.uuids = [u for u in (uuids or []) if u]
        self.active = active
        self.proc = None
        self.lines = []
        self.marks = []

    def _reader(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line))

    def __enter__(self):
        import threading
        if not self.active:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return self
        threading.Thread(target=self._reader, daemon=True).start()
        t0 = time.monotonic()
        while not self.lines and time.monotonic() - t0 < 10.0 and self.proc.poll() is None:
            time.sleep(0.02)
        return self

    def mark(self):
        """Start (first call) and end (second call) of the loaded window."""
        self.marks.append(time.monotonic())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        lo, hi = (self.marks + [float("inf")] * 2)[:2] if self.marks else (float("-inf"), float("inf"))
        rows = []
        for t, line in self.lines:
            if not lo <= t <= hi:
                continue
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            if self.uuids and not any(u in f[0] or f[0] in u for u in self.uuids):
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[4], f[5], f[6], f[7], f[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"], "samples": 0}
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[3:]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(rows), "gpus": len(self.uuids) or None,
                "window": "untimed replays of the same step around the timed region"}


# ---------------------------------------------------------- CPU path --
def cpu_reference_sample(seconds: float = 12.0, linears: int | None = None):
    """The reference's PyTorch path on the host cores over one layer's four
    linears (round robin) until `seconds` pass; returns (GB/s, cores, sample)."""
    import torch
    from oracle import fp8gq_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    ops = []
    for i, (name, K, N) in enumerate(SHAPES):
        x = torch.from_numpy(O.make_activation(1, K, seed=1000 + i)).bfloat16()
        wq, ws = O.make_weight(N, K, seed=2000 + i)
        ops.append((name, K, N, x, torch.from_numpy(wq).view(torch.float8_e4m3fn), torch.from_numpy(ws)))
    O.torch_reference_path(ops[0][3], ops[0][4], ops[0][5])        # warm
    done_bytes, t_total, n = 0, 0.0, 0
    while (linears is None and t_total < seconds) or (linears is not None and n < linears):
        name, K, N, x, w, s = ops[n % len(ops)]
        t0 = time.perf_counter()
        O.torch_reference_path(x, w, s)
        t_total += time.perf_counter() - t0
        done_bytes += alg_bytes(1, K, N)
        n += 1
    return done_bytes / t_total / 1e9, torch.get_num_threads(), \
        f"{n} linears of one Qwen3-8B layer (qkv, o, gate_up, down round robin), M=1, full path incl. weight dequant"


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    from oracle import fp8gq_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    ops = []
    for i, (name, K, N) in enumerate(SHAPES):
        x = torch.from_numpy(O.make_activation(1, K, seed=1000 + i)).bfloat16()
        wq, ws = O.make_weight(N, K, seed=2000 + i)
        ops.append((K, N, x, torch.from_numpy(wq).view(torch.float8_e4m3fn), torch.from_numpy(ws)))
    for j in range(args.warmup):
        K, N, x, w, s = ops[j % 4]
        O.torch_reference_path(x, w, s)
    t = 0.0
    total = 0
    for j in range(args.steps):
        K, N, x, w, s = ops[j % 4]
        t0 = time.perf_counter()
        O.torch_reference_path(x, w, s)
        t += time.perf_counter() - t0
        total += alg_bytes(1, K, N)
    gbs = total / t / 1e9
    cores = torch.get_num_threads()
    sample = ("one linear of a Qwen3-8B layer per step (qkv, o, gate_up, down round robin), M=1, "
              "torch CPU: group quant, dequant, fp32 matmul, bf16 out")
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 accumulate, bf16 out",
            "data": "synthetic (seeded)",
            "config": {"workload": WORKLOAD, "sample": sample, "M": 1},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------- GPU path --
def make_weight_gpu(N, K, seed, dev):
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.02).bfloat16().float()
    blk = w.view(N // 128, 128, K // 128, 128)
    ws = blk.abs().amax(dim=(1, 3)).clamp_min(1e-10) / 448.0
    q = (blk / ws[:, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(N, K)
    return q.contiguous(), ws.contiguous()


def decode_chain(layers, dev, M=1):
    """The decode step as a chain over the stack's weights: qkv -> o (the
    first 4096 columns of qkv's output, an attention stand-in) -> gate_up ->
    down (SwiGLU of gate_up's output) -> the next layer's qkv, every input the
    previous linear's output.  Returns (fp8gq.Linear list, step input)."""
    import torch
    import fp8gq
    H = SHAPES[0][1]
    h = torch.randn(M, H, device=dev).bfloat16()
    x = h
    lins = []
    for lin in layers:
        (_, _, Nq, wqkv, sqkv, _, _, _), (_, _, _, wo, so, _, _, _), \
            (_, _, Ngu, wgu, sgu, _, _, _), (_, _, Nd, wd, sd, _, _, _) = lin
        qkv = torch.empty(M, Nq, dtype=torch.bfloat16, device=dev)
        o = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        gu = torch.empty(M, Ngu, dtype=torch.bfloat16, device=dev)
        d = torch.empty(M, Nd, dtype=torch.bfloat16, device=dev)
        lins += [fp8gq.Linear(x, wqkv, sqkv, qkv), fp8gq.Linear(qkv[:, :H], wo, so, o),
                 fp8gq.Linear(o, wgu, sgu, gu), fp8gq.Linear(gu, wd, sd, d, swiglu=True)]
        x = d
    return lins, h


def layer_parity(layer, world, rank, dev):
    """Checks one layer's gathered outputs on every rank against the oracle of
    the UNSHARDED linears (a checker only, outside every timed region): rank r
    holds rows [r*N/w, (r+1)*N/w) of each weight, so the full weight is the
    ranks' shards in rank order.  Rank 0 evaluates the oracle (CPU, float64)
    on that full weight and the layer's input; every rank then compares its own
    full output with it (the tile kernel's tolerance: 3 bf16 ulp of max |ref| +
    1e-3, and rtol 1e-2 / atol 1e-2 * RMS) and with rank 0's copy bit for bit."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from oracle import fp8gq_oracle as O
    ok, worst, same = True, 0.0, True
    for name, K, N, wq, ws, x, out, shard in layer:
        if world > 1:
            wfull = torch.empty(N, K, dtype=torch.uint8, device=dev)
            sfull = torch.empty(N // 128, K // 128, dtype=torch.float32, device=dev)
            dist.all_gather_into_tensor(wfull, wq.view(torch.uint8).contiguous())
            dist.all_gather_into_tensor(sfull, ws.contiguous())
        else:
            wfull, sfull = wq.view(torch.uint8), ws
        exact = torch.zeros(1, N, dtype=torch.float64, device=dev)
        if rank == 0:
            _, ex, _, _ = O.fused_gemv_quant(x.float().cpu().numpy(), wfull.cpu().numpy(), sfull.cpu().numpy())
            exact.copy_(torch.from_numpy(ex))
        ref0 = out.clone()
        if world > 1:
            dist.broadcast(exact, src=0)
            dist.broadcast(ref0, src=0)
        ex = exact.cpu().numpy()
        got = out.float().cpu().numpy().astype(np.float64)
        atol = O.ref_atol(ex, 3.0)
        ok = ok and bool(O.rms_tolerance_ok(got, ex)) and bool(np.all(np.abs(got - ex) <= atol))
        worst = max(worst, float(np.abs(got - ex).max() / O.bf16_ulp_at(float(np.abs(ex).max()))))
        same = same and torch.equal(ref0, out)
    flags = torch.tensor([1.0 if ok else 0.0, 1.0 if same else 0.0, -worst], device=dev)
    if world > 1:
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    return {"linears": len(layer), "ok": bool(flags[0].item() == 1.0 and flags[1].item() == 1.0),
            "within_tolerance": bool(flags[0].item() == 1.0), "ranks_identical": bool(flags[1].item() == 1.0),
            "max_err_ulp": round(-float(flags[2].item()), 3), "ranks_checked": world,
            "against": "oracle of the unsharded linears (CPU, float64), layer 0 of the step, 3 bf16 ulp + "
                       "rtol 1e-2 / atol 1e-2*RMS"}


def paired_layer_parity(layer, world, rank, dev, h_in, res_in, norm_w, slabs0, slabs1, res1, res2, q_cols):
    """Paired tensor parallelism, layer 0 (a checker only, outside every timed
    region): every rank checks its own stages against the oracle -- the
    column-parallel qkv and gate_up slices within 3 bf16 ulp (and rtol 1e-2 /
    atol 1e-2 * RMS), the new residuals bit for bit, the row-parallel o and
    down partials within 3 ulp of the oracle of their K slice -- and the slabs
    every rank received must be identical on every rank."""
    import numpy as np
    import torch
    import torch.distributed as dist
    from oracle import fp8gq_oracle as O
    f32 = lambda t: t.float().cpu().numpy()  # noqa: E731
    u8 = lambda t: t.view(torch.uint8).cpu().numpy()  # noqa: E731
    (_, _, _, wqkv, sqkv, _, _, qkv_o), (_, _, _, wo, so, _, _, _), \
        (_, _, _, wgu, sgu, _, _, gu_o), (_, _, _, wd, sd, _, _, _) = layer
    worst, ok, exact_res = 0.0, True, True

    def within(got, exact):
        nonlocal worst, ok
        g = f32(got).astype(np.float64)
        worst = max(worst, float(np.abs(g - exact).max() / O.bf16_ulp_at(float(np.abs(exact).max()))))
        ok = ok and bool(O.rms_tolerance_ok(g, exact)) and bool(np.all(np.abs(g - exact) <= O.ref_atol(exact, 3.0)))

    _, ex, _, _, r = O.fused_add_rmsnorm_gemv_quant(f32(h_in), f32(res_in), f32(norm_w), u8(wqkv), f32(sqkv))
    within(qkv_o, ex)
    exact_res = exact_res and bool(np.array_equal(f32(res1), r))
    within(slabs0[rank], O.fused_gemv_quant(f32(qkv_o[:, :q_cols]), u8(wo), f32(so))[1])
    _, ex, _, _, r = O.fused_reduce_add_rmsnorm_gemv_quant([f32(slabs0[q]) for q in range(world)], f32(res1),
                                                           f32(norm_w), u8(wgu), f32(sgu))
    within(gu_o, ex)
    exact_res = exact_res and bool(np.array_equal(f32(res2), r))
    within(slabs1[rank], O.fused_swiglu_q_gemm(f32(gu_o), u8(wd), f32(sd))[1])
    same = True
    for t in (slabs0, slabs1, res1, res2):
        ref = t.clone()
        dist.broadcast(ref, src=0)
        same = same and torch.equal(ref, t)
    flags = torch.tensor([1.0 if ok else 0.0, 1.0 if exact_res else 0.0, 1.0 if same else 0.0, -worst], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    return {"linears": 4, "ok": bool(flags[0].item() == 1.0 and flags[1].item() == 1.0 and flags[2].item() == 1.0),
            "within_tolerance": bool(flags[0].item() == 1.0), "residuals_exact": bool(flags[1].item() == 1.0),
            "ranks_identical": bool(flags[2].item() == 1.0), "max_err_ulp": round(-float(flags[3].item()), 3),
            "ranks_checked": world,
            "against": "oracle per rank: column-parallel slices (add + RMSNorm prologue over the rank-ordered sum "
                       "of the slabs) and row-parallel partials of the K slice, layer 0, 3 bf16 ulp + rtol 1e-2 / "
                       "atol 1e-2*RMS; residuals bit-exact; slabs identical on every rank"}


def stack_runner_line(layers, dev, graph_us):
    """The decode chain as one persistent launch (fp8gq.StackRunner) against
    the same chain as 144 routed per-linear launches (CUDA graph of each)."""
    import torch
    import fp8gq
    lins, _ = decode_chain(layers, dev)
    runner = fp8gq.StackRunner(lins)
    runner.run()

    def per_linear():
        for lin in lins:
            if lin.swiglu:
                fp8gq.fused_swiglu_q_gemm(lin.x, lin.w, lin.ws, out=lin.out)
            else:
                fp8gq.fused_gemv_quant(lin.x, lin.w, lin.ws, out=lin.out)
    per_linear()
    torch.cuda.synchronize()
    b = STEP_BYTES + LAYERS * 2 * 12288        # the SwiGLU input of down is [gate | up]
    us_stack = graph_us([runner.run], reps=100)
    us_lin = graph_us([per_linear], reps=100)
    assert fp8gq.device_error() == 0, "a kernel recorded a wait timeout"
    return {"us_per_step": round(us_stack, 2), "gbs": round(b / (us_stack * 1e-6) / 1e9, 1),
            "per_linear_launches_us_per_step": round(us_lin, 2),
            "per_linear_launches_gbs": round(b / (us_lin * 1e-6) / 1e9, 1), "bytes_per_step": b,
            "linears": len(lins), "launches_per_step": 1,
            "kernel": "stack_kernel (persistent, cooperative, one CTA per SM)"}


def run_ours(args):
    import torch
    import torch.distributed as dist

    import fp8gq

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    fp8gq.load()
    fp8gq.set_static_weights(bool(args.static_weights))

    def barrier():
        if world > 1:
            dist.barrier()

    paired = world > 1 and args.tp_mode == "paired"
    # chain: the tagged words of the tagged mode, the step's 144 linears in
    # one persistent launch (fp8gq.ChainRunner) instead of one launch each
    chain = world > 1 and args.tp_mode == "chain"
    tagged = world > 1 and args.tp_mode in ("tagged", "chain")
    # ---- operands: each rank owns rows [r*N/world, (r+1)*N/world) of every
    # linear (gather / nccl modes), or, paired, rows of qkv and gate_up and
    # columns [r*K/world, (r+1)*K/world) of o and down
    layers = []
    xs_len = sum(K for _, K, _ in SHAPES)
    out_len = sum(N for _, _, N in SHAPES)
    # two copies of the step's inputs and outputs: copy 0 is the one the timed
    # CUDA graph uses; the end-to-end loop alternates between them (see e2e)
    x_all2 = torch.empty(2, LAYERS, xs_len, dtype=torch.bfloat16, device=dev)
    out_all2 = torch.empty(2, LAYERS, out_len, dtype=torch.bfloat16, device=dev)
    x_all, out_all = x_all2[0], out_all2[0]
    shard_all = torch.empty(LAYERS, out_len // world, dtype=torch.bfloat16, device=dev)
    g = torch.Generator(device=dev).manual_seed(7)
    for L in range(LAYERS):
        lin = []
        xo = oo = so = 0
        for i, (name, K, N) in enumerate(SHAPES):
            Nr = N // world
            if paired and name in ("o", "down"):
                wq, ws = make_weight_gpu(N, K // world, seed=100000 * L + 1000 * i + rank, dev=dev)
            else:
                wq, ws = make_weight_gpu(Nr, K, seed=100000 * L + 1000 * i + rank, dev=dev)
            x = x_all[L, xo:xo + K].view(1, K)
            xv = torch.randn(1, K, generator=g, device=dev)
            ch = torch.randperm(K, generator=g, device=dev)[: round(0.01 * K)]
            xv[:, ch] *= 20.0
            x.copy_(xv.bfloat16())
            lin.append((name, K, N, wq, ws, x, out_all[L, oo:oo + N].view(1, N),
                        shard_all[L, so:so + Nr].view(1, Nr)))
            xo += K
            oo += N
            so += Nr
        layers.append(lin)
    torch.cuda.synchronize()

    pg = None
    if world > 1 and args.tp_mode == "gather":
        from fp8gq.dist import PeerGather
        pg = PeerGather(out_all2.view(-1))
        # descriptors of every linear's output slice, built once (each call
        # waits for the previous linear's slices, as a decoder's next linear
        # would for its input)
        descs = [[pg.descriptor(lin[i][6], rank * (lin[i][2] // world), True) for i in range(len(SHAPES))]
                 for lin in layers]
    def at_parity(t, base2, parity):
        """The view of base2[parity] at the place t has in base2[0]."""
        off = (t.data_ptr() - base2[0].data_ptr()) // t.element_size()
        return base2[parity].view(-1)[off:off + t.numel()].view(t.shape)

    if tagged:
        # Tagged words: the step is a chain -- layer L's qkv reads layer L-1's
        # down output (layer 0: the step input, bf16), o the first 4096
        # columns of qkv's output (the attention stand-in), gate_up o's
        # output, down the first 12288 columns of gate_up's output -- every
        # input a tagged output of the linear before it, polled word by word
        # by the kernel that reads it.  A decode kernel turns the last
        # output into the step's bf16 result.  Two copies of the words for the
        # pipelined end-to-end loop.
        from fp8gq.dist import PeerGather
        words2 = torch.zeros(2, LAYERS, out_len // 2, dtype=torch.int64, device=dev)
        pg = PeerGather(words2.view(-1), tagged=True)
        dec2 = torch.empty(2, 1, SHAPES[-1][2], dtype=torch.bfloat16, device=dev)

        def chain_io(q):
            """[(input, output words, waits for its input)] per linear, copy q."""
            io, prev = [], None
            for L, lin in enumerate(layers):
                outs, oo = [], 0
                for name, K, N in SHAPES:
                    outs.append(words2[q, L, oo // 2:(oo + N) // 2].view(1, N // 2))
                    oo += N
                ins = [at_parity(lin[0][5], x_all2, q) if prev is None else prev,
                       outs[0][:, :SHAPES[1][1] // 2], outs[1], outs[2][:, :SHAPES[3][1] // 2]]
                for i in range(len(SHAPES)):
                    io.append((ins[i], outs[i], not (L == 0 and i == 0)))
                prev = outs[3]
            return io
        tagged_io = [chain_io(0), chain_io(1)]
        tdescs = [[pg.descriptor(o, rank * (SHAPES[k % len(SHAPES)][2] // world), w)
                   for k, (_, o, w) in enumerate(io)] for io in tagged_io]
        if chain:
            # link k reads linear k - 1's words, except layer 0's qkv (the step
            # input); every link's input is the output of the one before it
            runners = []
            for io in tagged_io:
                links = []
                for k, (x, o, w) in enumerate(io):
                    lin = layers[k // len(SHAPES)][k % len(SHAPES)]
                    links.append(fp8gq.Link(x=x, w=lin[3], ws=lin[4], out=o, src=k - 1 if w else -1))
                runners.append(fp8gq.ChainRunner(links, gather=pg))
    if paired:
        # Paired tensor parallelism, layer by layer:
        #   qkv      column-parallel, add + RMSNorm prologue over the sum of the
        #            previous layer's down partials (layer 0: the step input)
        #   o        row-parallel on this rank's q columns of the qkv output (the
        #            attention output stand-in), partial -> every rank's slab
        #   gate_up  column-parallel (gate and up rows of the rank together),
        #            prologue sums the o partials + residual, RMSNorm
        #   down     row-parallel, SwiGLU of the local gate_up slice, partial ->
        #            every rank's slab
        from fp8gq.dist import PeerGather
        H = SHAPES[0][1]
        slab_buf = torch.zeros(LAYERS * 2 * world * H, dtype=torch.bfloat16, device=dev)
        pg = PeerGather(slab_buf)
        slabs = slab_buf.view(LAYERS, 2, world, 1, H)
        res_buf = torch.empty(LAYERS + 1, 2, 1, H, dtype=torch.bfloat16, device=dev)
        h_in = torch.randn(1, H, generator=g, device=dev).bfloat16()
        res_buf[0, 1].copy_(torch.randn(1, H, generator=g, device=dev).bfloat16())
        norm_w = (torch.randn(H, generator=g, device=dev) * 0.1 + 1).bfloat16()
        pdesc = [[pg.partial_descriptor(slabs[L, j]) for j in range(2)] for L in range(LAYERS)]
        wdesc = pg.wait_descriptor()
        q_cols = SHAPES[1][1] // world          # o_proj's K slice: this rank's attention heads

    def paired_step():
        for L, lin in enumerate(layers):
            (_, _, _, wqkv, sqkv, _, _, qkv_o), (_, _, _, wo, so, _, _, _), \
                (_, _, _, wgu, sgu, _, _, gu_o), (_, _, _, wd, sd, _, _, _) = lin
            # residuals: layer L's qkv prologue reads res_buf[L, 1] and writes
            # res_buf[L + 1, 0]; its gate_up prologue reads that and writes
            # res_buf[L + 1, 1] (res_buf[0, 1] is the step's input residual)
            if L == 0:
                fp8gq.fused_add_rmsnorm_gemv_quant(h_in, res_buf[0, 1], norm_w, wqkv, sqkv, out=qkv_o,
                                                   residual_out=res_buf[1, 0])
            else:
                pg.reduce_norm_linear(slabs[L - 1, 1], res_buf[L, 1], norm_w, wqkv, sqkv, qkv_o, res_buf[L + 1, 0],
                                      desc=wdesc)
            pg.linear_partial(qkv_o[:, :q_cols], wo, so, slabs[L, 0], desc=pdesc[L][0])
            pg.reduce_norm_linear(slabs[L, 0], res_buf[L + 1, 0], norm_w, wgu, sgu, gu_o, res_buf[L + 1, 1],
                                  desc=wdesc)
            pg.linear_partial(gu_o, wd, sd, slabs[L, 1], swiglu=True, desc=pdesc[L][1])
        pg.wait(slabs[LAYERS - 1, 1, rank])     # the step ends when the last partials have landed

    def step():
        if paired:
            paired_step()
            return
        if chain:
            runners[0].run()
            pg.decode(tagged_io[0][-1][1], dec2[0])
            return
        if tagged:
            io = tagged_io[0]
            for k, (x, o, w) in enumerate(io):
                lin = layers[k // len(SHAPES)][k % len(SHAPES)]
                pg.linear(x, lin[3], lin[4], o, desc=tdescs[0][k])
            pg.decode(io[-1][1], dec2[0])       # the step ends when the last slices have landed
            return
        for li, lin in enumerate(layers):
            for i, (name, K, N, wq, ws, x, out, shard) in enumerate(lin):
                if world == 1:
                    fp8gq.fused_gemv_quant(x, wq, ws, out=out)
                elif pg is not None:
                    pg.linear(x, wq, ws, out, desc=descs[li][i])
                else:
                    fp8gq.fused_gemv_quant(x, wq, ws, out=shard)
                    dist.all_gather_into_tensor(out.view(-1), shard.view(-1))
        if pg is not None:
            pg.wait(layers[-1][-1][6])      # the step ends when the last slices have landed

    def prepared_step_list(parity=0):
        """The same step as prepared launches (fp8gq.prepared): every call
        recorded once, the whole step issued by one C call per run; parity 1
        runs it on the second copy of the inputs and outputs.  None for the
        NCCL mode (its all-gathers are not library launches)."""
        plans = []
        if chain:
            return None             # two launches per step: nothing to prepare
        if tagged:
            io = tagged_io[parity]
            for k, (x, o, w) in enumerate(io):
                lin = layers[k // len(SHAPES)][k % len(SHAPES)]
                plans.append(pg.prepare_linear(x, lin[3], lin[4], o, desc=tdescs[parity][k]))
            plans.append(pg.prepare_decode(io[-1][1], dec2[parity]))
        elif paired:
            for L, lin in enumerate(layers):
                (_, _, _, wqkv, sqkv, _, _, qkv_o), (_, _, _, wo, so, _, _, _), \
                    (_, _, _, wgu, sgu, _, _, gu_o), (_, _, _, wd, sd, _, _, _) = lin
                if L == 0:
                    plans.append(fp8gq.prepare_fused_add_rmsnorm_gemv_quant(
                        h_in, res_buf[0, 1], norm_w, wqkv, sqkv, out=qkv_o, residual_out=res_buf[1, 0]))
                else:
                    plans.append(pg.prepare_reduce_norm_linear(slabs[L - 1, 1], res_buf[L, 1], norm_w, wqkv, sqkv,
                                                               qkv_o, res_buf[L + 1, 0], desc=wdesc))
                plans.append(pg.prepare_linear_partial(qkv_o[:, :q_cols], wo, so, slabs[L, 0], desc=pdesc[L][0]))
                plans.append(pg.prepare_reduce_norm_linear(slabs[L, 0], res_buf[L + 1, 0], norm_w, wgu, sgu, gu_o,
                                                           res_buf[L + 1, 1], desc=wdesc))
                plans.append(pg.prepare_linear_partial(gu_o, wd, sd, slabs[L, 1], swiglu=True, desc=pdesc[L][1]))
            plans.append(pg.prepare_wait(slabs[LAYERS - 1, 1, rank]))
        elif world == 1:
            for lin in layers:
                for (name, K, N, wq, ws, x, out, shard) in lin:
                    plans.append(fp8gq.prepare_fused_gemv_quant(at_parity(x, x_all2, parity), wq, ws,
                                                                out=at_parity(out, out_all2, parity)))
        elif pg is not None:
            for li, lin in enumerate(layers):
                for i, (name, K, N, wq, ws, x, out, shard) in enumerate(lin):
                    o = at_parity(out, out_all2, parity)
                    d = descs[li][i] if parity == 0 else pg.descriptor(o, rank * (N // world), True)
                    plans.append(pg.prepare_linear(at_parity(x, x_all2, parity), wq, ws, o, desc=d))
            plans.append(pg.prepare_wait(at_parity(layers[-1][-1][6], out_all2, parity)))
        else:
            return None
        return fp8gq.LaunchList(plans)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier()
    # the prepared form of the step must leave the same outputs as the calls
    prepared = prepared_step_list()
    prepared_same = None

    def step_outputs():
        """What a step leaves (tagged: the words' values, whose tags advance
        with every call, and the decoded result)."""
        if paired:
            return [res_buf.clone(), slab_buf.clone()]
        if tagged:
            from fp8gq.dist import untag
            return [untag(words2[0]), dec2[0].clone()]
        return [out_all.clone()]
    if prepared is not None:
        final = step_outputs()
        prepared.run()
        torch.cuda.synchronize()
        barrier()
        prepared_same = all(torch.equal(a, b) for a, b in zip(final, step_outputs()))
        if world > 1:
            f = torch.tensor([1.0 if prepared_same else 0.0], device=dev)
            dist.all_reduce(f, op=dist.ReduceOp.MIN)
            prepared_same = bool(f.item() == 1.0)
    # the outputs of the warm-up steps, checked before anything is timed
    if paired:
        parity = paired_layer_parity(layers[0], world, rank, dev, h_in, res_buf[0, 1], norm_w, slabs[0, 0],
                                     slabs[0, 1], res_buf[1, 0], res_buf[1, 1], q_cols)
    elif tagged:
        # layer 0 as bf16 (inputs and outputs decoded from their words), and
        # the words' sequence numbers: one per output, consecutive along the
        # chain, the same on every rank
        from fp8gq.dist import tags, untag
        io = tagged_io[0]
        dec_layer, seqs = [], []
        for i, (name, K, N, wq, ws, x, out, shard) in enumerate(layers[0]):
            xin, o, _ = io[i]
            xb = xin if xin.dtype == torch.bfloat16 else untag(xin)
            dec_layer.append((name, K, N, wq, ws, xb, untag(o), shard))
            tg = tags(o)
            seqs.append(int(tg.flatten()[0]) if bool((tg == tg.flatten()[0]).all()) else -1)
        parity = layer_parity(dec_layer, world, rank, dev)
        tag_ok = all(t > 0 for t in seqs) and all(seqs[i + 1] == seqs[i] + 1 for i in range(len(seqs) - 1))
        st = torch.tensor(seqs, dtype=torch.int64, device=dev)
        st0 = st.clone()
        dist.broadcast(st0, src=0)
        f = torch.tensor([1.0 if (tag_ok and torch.equal(st, st0)) else 0.0], device=dev)
        dist.all_reduce(f, op=dist.ReduceOp.MIN)
        parity["tags_consistent"] = bool(f.item() == 1.0)
        parity["ok"] = parity["ok"] and parity["tags_consistent"]
        parity["against"] += ("; tagged words decoded, every word of an output carrying one sequence number, "
                              "consecutive along the chain and equal on every rank")
    else:
        parity = layer_parity(layers[0], world, rank, dev)
    barrier()

    # the timed step: a CUDA graph of it, or the chain's two launches issued
    # as they are (a cooperative launch is not captured)
    if chain:
        graph = None
        replay = step
    else:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        replay = graph.replay
    for _ in range(3):
        replay()
    torch.cuda.synchronize()
    barrier()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    uuids = [uuid]
    if world > 1:
        uuids = [None] * world
        dist.all_gather_object(uuids, uuid)

    # the load window around the timed region: about 0.4 s of untimed replays
    # before it and 0.2 s after it, the same count on every rank (rank 0's)
    e_a, e_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_a.record()
    for _ in range(5):
        replay()
    e_b.record()
    torch.cuda.synchronize()
    est_ms = max(e_a.elapsed_time(e_b) / 5, 1e-3)
    n_window = torch.tensor([min(20000, int(400.0 / est_ms) + 1)], device=dev)
    if world > 1:
        dist.broadcast(n_window, src=0)
    n_pre = int(n_window.item())
    n_post = max(1, n_pre // 2)

    # ---- timed region: K steps (graph replays), CUDA events, max over ranks
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(uuids, active=rank == 0)
    nvc = NvlinkCounter(local) if world > 1 else None
    with sampler:
        barrier()
        torch.cuda.synchronize()
        sampler.mark()
        if nvc is not None:
            nvc.start()
        for _ in range(n_pre):
            replay()
        start.record()
        for _ in range(args.steps):
            replay()
        end.record()
        for _ in range(n_post):
            replay()
        torch.cuda.synchronize()
        nv_win = nvc.stop() if nvc is not None else None
        sampler.mark()
        barrier()
    ms = start.elapsed_time(end) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clocks = sampler.summary()
    nvlink = None
    if world > 1:
        # NVLink bytes per step, each rank's own counters over the loaded
        # window (every replay in it is the same step), against what the step
        # must send: each rank's output slices (or partials) to world - 1 peers
        n_win = n_pre + args.steps + n_post
        mine = [nv_win[0] / n_win, nv_win[1] / n_win] if nv_win is not None else [-1.0, -1.0]
        allv = [None] * world
        dist.all_gather_object(allv, (mine, nvc.error))
        nvc.close()
        if paired:
            alg = 2 * LAYERS * SHAPES[0][1] * 2 * (world - 1)
        elif pg is not None:
            alg = LAYERS * sum(N // world for _, _, N in SHAPES) * (4 if tagged else 2) * (world - 1)
        else:
            alg = None
        nvlink = {"tx_bytes_per_step": [round(v[0][0]) if v[0][0] >= 0 else None for v in allv],
                  "rx_bytes_per_step": [round(v[0][1]) if v[0][1] >= 0 else None for v in allv],
                  "algorithmic_tx_bytes_per_step": alg,
                  "source": "NVML GPM NVLINK_TOTAL_TX/RX_PER_SEC over the loaded window, per rank",
                  "errors": [v[1] for v in allv if v[1]] or None}
    value = STEP_BYTES / (ms * 1e-3) / 1e9
    launches = (2 if chain else LAYERS * len(SHAPES) + (1 if pg is not None else 0)) * args.steps

    # ---- per-linear device time: graph of the 36 launches of one shape
    def graph_us(calls, reps=20):
        g1 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g1):
            for c in calls:
                c()
        g1.replay()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(reps):
            g1.replay()
        s1.record()
        torch.cuda.synchronize()
        del g1
        return s0.elapsed_time(s1) * 1e3 / (reps * len(calls))

    def per_shape(kernel):
        """Device time per call of each shape's op on this rank's weights
        (graph of the 36 layers' launches).  Paired: o and down are the
        row-parallel ops on K / world columns (down with its SwiGLU prologue)."""
        res = {}
        for i, (name, K, N) in enumerate(SHAPES):
            rowpar = paired and name in ("o", "down")
            swiglu = paired and name == "down" and kernel == "auto"
            Kl, Nl = (K // world, N) if rowpar else (K, N // world)
            calls = []
            for lin in layers:
                _, _, _, wq, ws, x, out, shard = lin[i]
                o = out if (world == 1 or rowpar) else shard
                if swiglu:
                    gu = x[:, :2 * Kl]
                    calls.append(lambda gu=gu, wq=wq, ws=ws, o=o: fp8gq.fused_swiglu_q_gemm(gu, wq, ws, out=o))
                else:
                    xl = x[:, :Kl]
                    calls.append(lambda xl=xl, wq=wq, ws=ws, o=o: fp8gq.fused_gemv_quant(xl, wq, ws, out=o,
                                                                                         kernel=kernel))
            us = graph_us(calls)
            b = alg_bytes(1, Kl, Nl)
            res[name] = {"us_per_call": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1), "bytes_per_call": b}
            if kernel == "auto":
                res[name]["kernel"] = ROUTED_KERNEL(Nl, Kl, swiglu=swiglu)
        return res

    per = per_shape("auto")
    per_row = per_shape("row")
    per_tm = per_shape("tm")

    extra = {}
    if world == 1:
        extra["stack_runner"] = stack_runner_line(layers, dev, graph_us)
    if world == 1:
        # fused SwiGLU + quant + down_proj at M = 1 (gate_up output 24576 -> 4096)
        gus = [(torch.randn(1, 24576, device=dev) * 1.5).bfloat16() for _ in range(4)]
        calls = [lambda lin=lin, gu=gus[i % 4]: fp8gq.fused_swiglu_q_gemm(gu, lin[3][3], lin[3][4], out=lin[3][6])
                 for i, lin in enumerate(layers)]
        us = graph_us(calls)
        b = alg_bytes(1, 12288, 4096) + 2 * 12288
        extra["swiglu_down_m1"] = {"us_per_call": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1),
                                   "kernel": ROUTED_KERNEL(4096, 12288, swiglu=True)}
        # TM-blocked small batches on the Qwen3-4B shapes (weights rotate through
        # more than 4x the L2 so every call streams from HBM)
        tmb = {}
        for name, K, N in (("q", 2560, 4096), ("gate_up", 2560, 19456), ("down", 9728, 2560)):
            copies = max(4, -(-4 * 126 * 2**20 // (N * K)))
            wl = [make_weight_gpu(N, K, seed=500 + c, dev=dev) for c in range(copies)]
            for M in (2, 4, 8, 16):
                xm = torch.randn(M, K, device=dev).bfloat16()
                om = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
                calls = [lambda w=w: fp8gq.fused_gemv_quant(xm, w[0], w[1], out=om) for w in wl]
                us = graph_us(calls, reps=max(4, 200 // copies))
                b = alg_bytes(M, K, N)
                tmb[f"{name}_M{M}"] = {"us_per_call": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1)}
            del wl
        extra["tm_blocked_qwen3_4b"] = tmb
        # add + RMSNorm as the prologue of qkv and gate_up (M = 1), against the
        # norm as its own kernel followed by the linear
        nrm = {}
        hid = torch.randn(1, 4096, device=dev).bfloat16()
        resid = torch.randn(1, 4096, device=dev).bfloat16()
        nw = (torch.randn(4096, device=dev) * 0.1 + 1).bfloat16()
        hbuf = torch.empty(1, 4096, dtype=torch.bfloat16, device=dev)
        rbuf = torch.empty(1, 4096, dtype=torch.bfloat16, device=dev)
        for i, name in ((0, "qkv"), (2, "gate_up")):
            outs_ = [lin[i][6] for lin in layers]
            fused = [lambda lin=lin, o=o: fp8gq.fused_add_rmsnorm_gemv_quant(hid, resid, nw, lin[i][3], lin[i][4],
                                                                            out=o, residual_out=rbuf)
                     for lin, o in zip(layers, outs_)]

            def unfused_call(lin, o):
                fp8gq.add_rmsnorm(hid, resid, nw, out=hbuf, residual_out=rbuf)
                fp8gq.fused_gemv_quant(hbuf, lin[i][3], lin[i][4], out=o)
            unfused = [lambda lin=lin, o=o: unfused_call(lin, o) for lin, o in zip(layers, outs_)]
            nrm[name] = {"fused_us": round(graph_us(fused), 3), "norm_then_linear_us": round(graph_us(unfused), 3)}
        extra["add_rmsnorm_prologue_m1"] = nrm
        # lm_head of Qwen3-8B (151936 x 4096, 622 MB of e4m3), two weight copies
        lm = [make_weight_gpu(151936, 4096, seed=900 + c, dev=dev) for c in range(2)]
        lmh = {}
        for M in (1, 4):
            xm = torch.randn(M, 4096, device=dev).bfloat16()
            om = torch.empty(M, 151936, dtype=torch.bfloat16, device=dev)
            calls = [lambda w=w: fp8gq.fused_gemv_quant(xm, w[0], w[1], out=om) for w in lm]
            us = graph_us(calls, reps=20)
            b = alg_bytes(M, 4096, 151936)
            lmh[f"M{M}"] = {"us_per_call": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1), "bytes_per_call": b}
        extra["lm_head_qwen3_8b"] = lmh
        del lm
        torch.cuda.empty_cache()
        # stand-alone SwiGLU + quant writer on a prefill chunk (512 tokens x
        # Qwen3-4B intermediate 9728), gate/up rotating through > L2
        wr = []
        for c in range(8):
            gw = torch.randn(512, 2 * 9728, device=dev).bfloat16()
            wr.append((gw[:, :9728], gw[:, 9728:]))
        calls = [lambda p=p: fp8gq.fused_swiglu_quant(p[0], p[1]) for p in wr]
        us = graph_us(calls)
        b = 2 * 512 * 9728 * 2 + 512 * 9728 + 4 * 512 * 76
        extra["swiglu_quant_writer_512x9728"] = {"us_per_call": round(us, 3), "gbs": round(b / (us * 1e-6) / 1e9, 1),
                                                 "bytes_per_call": b}
        del wr
        torch.cuda.empty_cache()

    peak, peak_kind = measured_peak()
    gu = per["gate_up"]
    roofline = {"bound": "hbm", "achieved": gu["gbs"], "peak": peak, "unit": "GB/s",
                "frac": round(gu["gbs"] / peak, 4),
                "traffic": NCU_TRAFFIC_BYTES.get(gu["kernel"]) if world == 1 else None,
                "kernel": "%s (gate_up 4096->24576%s)" % (
                    gu["kernel"], f", N/{world} rows per rank" if world > 1 else ""),
                "peak_source": f"{peak_kind} hbm_gbs (copy bandwidth)"}

    # ---- e2e: public API, eager, host buffers in and out
    # (paired: the step's input hidden state and residual in, the last
    # layer's down partials and residual out; otherwise every linear's input
    # in and every output out)
    # (tagged: the step's input in, its decoded result out -- the chain
    # carries everything else)
    if tagged:
        e2e_in, e2e_out = [layers[0][0][5]], [dec2[0]]
    else:
        e2e_in = [h_in, res_buf[0, 1]] if paired else [x_all]
        e2e_out = [slabs[LAYERS - 1, 1], res_buf[LAYERS, 1]] if paired else [out_all]
    hosts_in = [torch.empty_like(t, device="cpu").pin_memory() for t in e2e_in]
    for t, h in zip(e2e_in, hosts_in):
        h.copy_(t.cpu())
    hosts_out = [torch.empty_like(t, device="cpu").pin_memory() for t in e2e_out]
    def e2e_ms_of(run_step, copies=True):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for it in range(3 + args.e2e_steps):
            if it == 3:
                barrier()
                torch.cuda.synchronize()
                e0.record()
            if copies:
                for t, h in zip(e2e_in, hosts_in):
                    t.copy_(h, non_blocking=True)
            if run_step is not None:
                run_step()
            if copies:
                for t, h in zip(e2e_out, hosts_out):
                    h.copy_(t, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        ms_ = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            t = torch.tensor([ms_], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_ = float(t.item())
        return ms_

    def e2e_pipelined_ms(graphs=False):
        """The prepared step with the copies overlapped, through two copies of
        the step's buffers: step k runs on copy k % 2, its inputs are copied in
        (one stream) while step k - 1 runs, and its outputs copied out (another
        stream) while step k + 1 runs.  The compute stream waits twice per step
        -- for its inputs before the first layer, and before the last layer for
        the copy out of step k - 1 (same copy as step k + 1), which is also the
        point after which the other ranks may store step k + 1's slices into
        it -- so the chain of launches is not broken at every layer.  Every
        step's copies, in and out, are inside the timed region.  With graphs,
        each half of the step (its launch lists as they are) is captured once
        into a CUDA graph and replayed, as a serving loop replays its decode
        step: eager launches cost the device more per launch than replayed
        ones."""
        if paired or prepared is None:
            return None
        npl = len(SHAPES)
        lists = []
        for parity in (0, 1):
            full = prepared if parity == 0 else prepared_step_list(1)
            head = fp8gq.LaunchList(full.plans[:npl * (LAYERS - 1)])
            tail = fp8gq.LaunchList(full.plans[npl * (LAYERS - 1):])
            if graphs:
                gh, gt = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                with torch.cuda.graph(gh):
                    head.run()
                with torch.cuda.graph(gt):
                    tail.run()
                lists.append((gh, gt))
            else:
                lists.append((head, tail))
        comp = torch.cuda.current_stream(dev)
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        in_ready = [torch.cuda.Event(), torch.cuda.Event()]
        step_done = [torch.cuda.Event(), torch.cuda.Event()]
        out_free = [torch.cuda.Event(), torch.cuda.Event()]
        h_in, h_out = hosts_in[0], hosts_out[0]
        start_gate = torch.cuda.Event()

        def enqueue(k, gate=None):
            q = k % 2
            with torch.cuda.stream(s_in):
                if gate is not None:
                    s_in.wait_event(gate)
                if k >= 2:
                    s_in.wait_event(step_done[q])        # step k - 2 is done with copy q's inputs
                (at_parity(layers[0][0][5], x_all2, q) if tagged else x_all2[q]).copy_(h_in, non_blocking=True)
                in_ready[q].record(s_in)
            comp.wait_event(in_ready[q])
            head, tail = lists[q]
            head.replay() if graphs else head.run()
            if k >= 1:
                comp.wait_event(out_free[(k - 1) % 2])   # step k - 1's outputs are copied out
            tail.replay() if graphs else tail.run()
            step_done[q].record(comp)
            with torch.cuda.stream(s_out):
                s_out.wait_event(step_done[q])
                h_out.copy_(dec2[q] if tagged else out_all2[q], non_blocking=True)
                out_free[q].record(s_out)

        for k in range(2):                               # fill the pipeline
            enqueue(k)
        comp.wait_event(out_free[1])
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(comp)
        start_gate.record(comp)
        for k in range(2, 2 + args.e2e_steps):
            enqueue(k, gate=start_gate if k == 2 else None)
        comp.wait_event(out_free[(1 + args.e2e_steps) % 2])
        e1.record(comp)
        torch.cuda.synchronize()
        ms_ = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            t = torch.tensor([ms_], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_ = float(t.item())
        return ms_

    eager_ms = e2e_ms_of(step)
    serial_ms = e2e_ms_of(prepared.run) if prepared is not None else eager_ms
    piped_eager_ms = e2e_pipelined_ms()
    piped_ms = e2e_pipelined_ms(graphs=True)
    e2e_ms = piped_ms if piped_ms is not None else serial_ms
    # where the end-to-end time goes: the same loop without the copies, and
    # the copies alone
    parts_ms = {"without_copies": e2e_ms_of(prepared.run if prepared is not None else step, copies=False),
                "copies_alone": e2e_ms_of(None)}
    e2e = {"value": round(STEP_BYTES / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
           "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in e2e_in),
           "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in e2e_out),
           "ms_per_step": round(e2e_ms, 4),
           "path": (("fp8gq.LaunchList of prepared " + ("PeerGather paired linears" if paired else
                                                          "PeerGather.prepare_linear calls on tagged words "
                                                          "(the step input in, the decoded result out)" if tagged else
                                                          "PeerGather.prepare_linear calls" if pg is not None else
                                                          "fp8gq.prepare_fused_gemv_quant calls") +
                     (", two copies of the step's buffers: each step's inputs copied in while the step before "
                      "runs and its outputs copied out while the step after runs, on two copy streams; each half "
                      "of the step captured once into a CUDA graph and replayed" if piped_ms is not None else
                      ", one run per step, copies before and after it (eager, no graph)"))
                    if prepared is not None else
                    "fp8gq.ChainRunner.run + PeerGather.decode per step (two launches), the step input in and the "
                    "decoded result out" if chain else "fp8gq.fused_gemv_quant (eager) per linear + NCCL all-gather"),
           "eager_pipelined": ({"ms_per_step": round(piped_eager_ms, 4),
                                "value": round(STEP_BYTES / (piped_eager_ms * 1e-3) / 1e9, 3),
                                "path": "the same pipelined loop with the launch lists issued eagerly (no graph)"}
                               if piped_eager_ms is not None else None),
           "serial_copies": {"ms_per_step": round(serial_ms, 4),
                             "value": round(STEP_BYTES / (serial_ms * 1e-3) / 1e9, 3)},
           "prepared_matches_calls": prepared_same,
           "parts_ms_per_step": {k: round(v, 4) for k, v in parts_ms.items()},
           "eager_calls": {"ms_per_step": round(eager_ms, 4),
                           "value": round(STEP_BYTES / (eager_ms * 1e-3) / 1e9, 3),
                           "path": ("fp8gq.dist.PeerGather paired linears (eager)" if paired else
                                    "fp8gq.ChainRunner.run + PeerGather.decode" if chain else
                                    "fp8gq.dist.PeerGather.linear (eager)" if pg is not None else
                                    "fp8gq.fused_gemv_quant (eager) per linear")}}

    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0, "a kernel recorded a wait timeout"
    del graph
    barrier()
    if pg is not None:
        pg.close()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_reference_sample()
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "e4m3 x e4m3 -> fp32 accumulate, bf16 out", "data": "synthetic (seeded)",
                "config": {"workload": WORKLOAD, "M": 1, "layers": LAYERS,
                           "bytes_per_step": STEP_BYTES,
                           "l2": "inputs larger than L2 (6.95 GB of weights per step, 126 MB L2)",
                           "parallelism": ((f"paired tensor parallel x{world}: qkv, gate_up column-parallel, "
                                            "o, down row-parallel; partials stored into every rank's slab by "
                                            "the kernels over NVLink and summed in the next linear's add + "
                                            "RMSNorm prologue") if paired else
                                           (f"N-sharded x{world}, the step's 144 linears in one persistent "
                                            "cooperative launch (fp8gq.ChainRunner), output slices stored into "
                                            "every rank over NVLink as tagged words, each linear polling the "
                                            "previous one's") if chain else
                                           (f"N-sharded x{world}, output slices stored into every rank by the "
                                            "kernels over NVLink as tagged words (each linear reading the "
                                            "previous one's output: qkv -> o -> gate_up -> down -> next qkv), "
                                            "no flags") if tagged else
                                           (f"N-sharded x{world}, output slices stored into every rank by the "
                                            "kernels over NVLink") if pg is not None else
                                           f"N-sharded x{world} + NCCL all-gather per linear") if world > 1
                           else "single GPU",
                           "timing": ("the step's two launches (chain, decode) issued as they are, CUDA events"
                                      if chain else "CUDA graph of one step, CUDA events"),
                           "static_weights": bool(args.static_weights)},
                "us_per_call": {k: v["us_per_call"] for k, v in per.items()},
                "per_linear": per, "per_linear_row_kernel": per_row, "per_linear_tile_kernel": per_tm, **extra,
                "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "parity": parity, "nvlink": nvlink,
                "gpu_launches": launches, "clocks": clocks}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_profile_case(args):
    """One linear of the stack, launched back to back; no timing, no output
    checks.  Used as the command under ncu."""
    import torch
    import fp8gq
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    fp8gq.load()
    if args.profile_case == "stack":
        # the decode step's 144 routed linears (36 layers x 4 shapes), eager
        lin = []
        g = torch.Generator(device=dev).manual_seed(2)
        for L in range(LAYERS):
            for i, (name, K, N) in enumerate(SHAPES):
                wq, ws = make_weight_gpu(N, K, seed=100000 * L + 1000 * i, dev=dev)
                lin.append((torch.randn(1, K, generator=g, device=dev).bfloat16(), wq, ws))
        for _ in range(args.warmup + args.steps):
            for x, wq, ws in lin:
                fp8gq.fused_gemv_quant(x, wq, ws)
        torch.cuda.synchronize()
        assert fp8gq.device_error() == 0
        print(json.dumps({"profile_case": "stack", "launches": (args.warmup + args.steps) * len(lin),
                          "bytes_per_step": STEP_BYTES}))
        return
    if args.profile_case.startswith("stack_runner"):
        # the decode chain of L layers (default 4: 772 MB of weights, > L2)
        # as one persistent launch per step
        nl = int(args.profile_case.split("L=")[1]) if "L=" in args.profile_case else 4
        layers = []
        for L in range(nl):
            lin = []
            for i, (name, K, N) in enumerate(SHAPES):
                wq, ws = make_weight_gpu(N, K, seed=100000 * L + 1000 * i, dev=dev)
                lin.append((name, K, N, wq, ws, None, None, None))
            layers.append(lin)
        lins, _ = decode_chain(layers, dev)
        runner = fp8gq.StackRunner(lins)
        for _ in range(args.warmup + args.steps):
            runner.run()
        torch.cuda.synchronize()
        assert fp8gq.device_error() == 0
        print(json.dumps({"profile_case": args.profile_case, "launches": args.warmup + args.steps,
                          "bytes_per_launch": nl * sum(alg_bytes(1, K, N) for _, K, N in SHAPES) + nl * 2 * 12288}))
        return
    parts = args.profile_case.split(":")
    shape, kernel, M = parts[0], "auto", 1
    for p in parts[1:]:
        if p.startswith("M="):
            M = int(p[2:])
        else:
            kernel = p
    g = torch.Generator(device=dev).manual_seed(2)
    if shape in ("writer", "add_rmsnorm", "group_quant"):
        # the activation-side kernels on their own, M rows of Qwen3-8B widths
        # (writer: intermediate 12288, the others: hidden 4096)
        if shape == "writer":
            gu = torch.randn(M, 2 * 12288, generator=g, device=dev).bfloat16()
            gate, up = gu[:, :12288], gu[:, 12288:]
            fn = lambda: fp8gq.fused_swiglu_quant(gate, up)  # noqa: E731
            nbytes = M * 12288 * (4 + 1) + 4 * M * 96
        elif shape == "add_rmsnorm":
            h = torch.randn(M, 4096, generator=g, device=dev).bfloat16()
            r = torch.randn(M, 4096, generator=g, device=dev).bfloat16()
            nw = (torch.randn(4096, generator=g, device=dev) * 0.1 + 1).bfloat16()
            o, ro = torch.empty_like(h), torch.empty_like(h)
            fn = lambda: fp8gq.add_rmsnorm(h, r, nw, out=o, residual_out=ro)  # noqa: E731
            nbytes = M * 4096 * 2 * 4 + 4096 * 2
        else:
            h = torch.randn(M, 4096, generator=g, device=dev).bfloat16()
            fn = lambda: fp8gq.group_quant(h)  # noqa: E731
            nbytes = M * 4096 * (2 + 1) + 4 * M * 32
        for _ in range(args.warmup + args.steps):
            fn()
        torch.cuda.synchronize()
        assert fp8gq.device_error() == 0
        print(json.dumps({"profile_case": args.profile_case, "launches": args.warmup + args.steps,
                          "bytes_per_launch": nbytes}))
        return
    dims = {n: (K, N) for n, K, N in SHAPES}
    dims["swiglu_down"] = (12288, 4096)
    if shape.startswith("norm_"):
        dims[shape] = dims[shape[5:]]
    K, N = dims[shape]
    wq, ws = make_weight_gpu(N, K, seed=1, dev=dev)
    if shape.startswith("norm_"):
        # add + RMSNorm as the prologue of the linear
        h = torch.randn(M, K, generator=g, device=dev).bfloat16()
        r = torch.randn(M, K, generator=g, device=dev).bfloat16()
        nw = (torch.randn(K, generator=g, device=dev) * 0.1 + 1).bfloat16()
        fn = lambda: fp8gq.fused_add_rmsnorm_gemv_quant(h, r, nw, wq, ws)  # noqa: E731
    elif shape == "swiglu_down":
        x = (torch.randn(M, 2 * K, generator=g, device=dev) * 1.5).bfloat16()
        fn = lambda: fp8gq.fused_swiglu_q_gemm(x, wq, ws)  # noqa: E731
    else:
        x = torch.randn(M, K, generator=g, device=dev).bfloat16()
        fn = lambda: fp8gq.fused_gemv_quant(x, wq, ws, kernel=kernel)  # noqa: E731
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    assert fp8gq.device_error() == 0
    print(json.dumps({"profile_case": args.profile_case, "launches": args.warmup + args.steps,
                      "bytes_per_launch": alg_bytes(M, K, N)}))


def main():
    args = parse()
    if args.profile_case:
        run_profile_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
