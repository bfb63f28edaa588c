"""Benchmark: LaplaceSubtraction forward+backward (Gdist/s) on the pyramid-ViT
stage-1 shape, with the batched NewtonInverse (matrices/s), the long-sequence
configuration 5 and the configuration-4 attention block reported beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One process per GPU (torchrun for N > 1).  The headline path shards over B*H
with no collective: every rank runs its own batch-32 slice of a global batch
32*N (weak scaling).  A step is one pass of the hot path over one batch: S =
LaplaceSub(Q, K^T), then both gradients (dQ, dK^T) of an upstream dS, through
the C ABI with inputs resident in HBM.  Timing: W untimed steps, then K steps
bracketed by a barrier and cudaDeviceSynchronize; each step is timed with CUDA
events on the launching stream and an L2 flush (a 256 MB write, outside the
events) separates steps; a GPU sleep enqueued ahead of the timed steps lets
the host queue them all, so host launch jitter never shows up as device time;
the max over ranks is reported, and the per-rank figures are listed.  Rank 0
prints one JSON line.

Sub-records of the same line:
* ``newton_inverse`` — configuration 3 (4096 x 128^2, 12 iterations) with
  the scaled-transpose init in split3 and mixed arithmetic, and the drop-in
  NewtonInverse_forward (reference init, A + 0.01 I, split3);
* ``config5`` — the north-star long-sequence workload (B=8, H=16, N=16384,
  D=64, M=256, bf16 LaplaceSub fwd+bwd + the 256x256 landmark inverse x10)
  strong-scaled over the ranks; with N > 1 dQ, dK^T and X are replicated on
  every rank by the kernels' own stores into the other GPUs' gather buffers
  (NVLink peer memory), with the NCCL all-gather after the compute timed
  beside it;
* ``config4`` — the Laplacian attention block fwd+bwd, bf16 [128,8,196,64],
  M = 49, 8 iterations (rank 0 of a 1-GPU run).

--impl reference times the reference's own operators (compiled from its
sources for sm_100 into oracle/_ref by oracle/build_ref.py) on the same
workload; under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "LaplaceSub Gdist/s & NewtonInverse matrices/s at 1/2/4/8 B200 vs roofline"
UNIT = "Gdist/s"


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self._stop = threading.Event()
        self._th = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._th = threading.Thread(target=self._run, daemon=True)
        self._th.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._th:
            self._th.join(timeout=10)

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            if len(r) > 8:
                for nm, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def _flush_buffer(dev):
    return torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)


def time_steps(step, steps, warmup, flush, stream, prefill_ms=None):
    """Warm up, then time `steps` calls of step() with events on `stream`.

    A GPU sleep is enqueued before the timed steps so that the host has queued
    them all before the GPU reaches them (outside the events): host launch
    cost then cannot show up as device time.  If the sleep had already ended
    when the host finished queueing (the GPU waited on the host), the loop is
    repeated with a sleep twice as long, up to four times."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if prefill_ms is None:
        prefill_ms = 4.0 + 1.0 * steps  # ~1 ms of host time per step, generous
    for attempt in range(4):
        if torch.distributed.is_initialized():
            torch.distributed.barrier()
        torch.cuda.synchronize()
        done = torch.cuda.Event()
        if prefill_ms > 0:
            torch.cuda._sleep(int(prefill_ms * 2.0e6))  # ~2 GHz SM clock
        done.record(stream)
        evs = []
        for _ in range(steps):
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            step()
            b.record(stream)
            evs.append((a, b))
        starved = prefill_ms > 0 and done.query()
        torch.cuda.synchronize()
        if torch.distributed.is_initialized():
            flag = torch.tensor([1.0 if starved else 0.0], device=torch.device("cuda", torch.cuda.current_device()))
            torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX)
            starved = bool(flag.item() > 0)
        if not starved or prefill_ms <= 0:
            break
        prefill_ms *= 2
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    return [a.elapsed_time(b) for a, b in evs]


def per_rank(values):
    """All ranks' values of a few floats (list per rank); [values] on one process."""
    if not torch.distributed.is_initialized():
        return [list(values)]
    world = torch.distributed.get_world_size()
    t = torch.tensor(list(values), dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
    out = [torch.empty_like(t) for _ in range(world)]
    torch.distributed.all_gather(out, t)
    return [[round(float(x), 5) for x in o.tolist()] for o in out]


def max_over_ranks(x: float) -> float:
    if not torch.distributed.is_initialized():
        return x
    t = torch.tensor([x], dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def laplace_bytes(bh, n, m, d, es):
    fwd = es * (bh * n * d + bh * d * m + bh * n * m)
    bwd = es * (bh * n * m + bh * n * d + bh * d * m + bh * n * d + bh * d * m)
    return fwd, bwd


def cpu_baseline_laplace(w, threads):
    """Oracle (C port of the reference arithmetic) on host threads, on a
    bounded sample of (b,h) slices of the same workload."""
    import numpy as np

    from oracle import oracle as O

    O.set_threads(threads)
    q = w["q"].cpu().numpy()
    k = w["kT"].cpu().numpy()
    g = w["ds"].cpu().numpy()
    B, H, N, D = q.shape
    M = k.shape[-1]
    sample_bh = 0
    t0 = time.perf_counter()
    b = 0
    while True:
        qs, ks, gs = q[b:b + 1], k[b:b + 1], g[b:b + 1]
        O.laplace_fwd(qs, ks)
        O.laplace_bwd_query(gs, qs, ks)
        O.laplace_bwd_key(gs, qs, ks)
        sample_bh += H
        b += 1
        el = time.perf_counter() - t0
        if el > 10.0 or b >= B:
            break
    value = sample_bh * N * M / el / 1e9
    return {"value": value, "unit": UNIT, "cores": O.threads(), "kind": "port",
            "sample": f"{sample_bh} of {B * H} (b,h) slices of the same workload (fwd + dQ + dK), "
                      f"{el:.1f} s on {O.threads()} host threads, oracle/oracle.c"}


def cpu_baseline_eager(w, threads, budget_s=8.0):
    """The reference semantics in PyTorch eager on the host cores (the form the
    north star names): S = cdist_1(Q, L), dQ = sum_j dS sign(Q - L_j), dK^T =
    -sum_i dS sign(Q_i - L), over a bounded sample of (b,h) slices."""
    torch.set_num_threads(threads)
    q = w["q"].cpu().float()
    kT = w["kT"].cpu().float()
    g = w["ds"].cpu().float()
    B, H, N, D = q.shape
    M = kT.shape[-1]
    done = 0
    t0 = time.perf_counter()
    for b in range(B):
        for h in range(H):
            qs, L, gs = q[b, h], kT[b, h].t().contiguous(), g[b, h]
            torch.cdist(qs[None], L[None], p=1)
            for r0 in range(0, N, 512):  # bounded intermediate [512, M, D]
                sg = torch.sign(qs[r0:r0 + 512, None, :] - L[None, :, :])
                gr = gs[r0:r0 + 512, :, None]
                (gr * sg).sum(1)
                (gr * sg).sum(0)
            done += 1
            if time.perf_counter() - t0 > budget_s:
                break
        if time.perf_counter() - t0 > budget_s:
            break
    el = time.perf_counter() - t0
    return {"value": done * N * M / el / 1e9, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{done} of {B * H} (b,h) slices, PyTorch eager fp32 on the host (cdist p=1 + sign sums), "
                      f"{el:.1f} s"}


def packed_fp16_record(dev, steps, warmup, flush, stream, issue_peak):
    """Configuration 2 forward in fp16: the bit-exact kernel (fp32 arithmetic,
    2 FP32 instructions per term) beside the opt-in packed-half2 kernel (one
    HSUB2 + one HADD2 per two terms), with its largest relative error against
    the bit-exact result on the same inputs."""
    from laplacianformer_b200 import capi, workloads

    w = workloads.config2(device=dev, dtype=torch.float16)
    q, kT = w["q"], w["kT"]
    B, H, N, D = q.shape
    M = kT.shape[-1]
    terms = B * H * N * M * D
    s_exact = torch.empty(B, H, N, M, device=dev, dtype=torch.float16)
    s_packed = torch.empty_like(s_exact)
    out = {}
    for name, fn, s_out in (("exact", capi.laplace_sub_fwd, s_exact), ("packed", capi.laplace_sub_fwd_packed, s_packed)):
        ms = statistics.mean(time_steps(lambda: fn(q, kT, s_out), steps, warmup, flush, stream))
        out[name] = {"ms": ms, "gterms_per_s": terms / (ms / 1e3) / 1e9,
                     "kernel": "lsub_fwd_kernel<__half>" if name == "exact" else "lsub_fwd_h2_kernel"}
    torch.cuda.synchronize()
    rel = ((s_packed.float() - s_exact.float()).abs() / s_exact.float().abs().clamp_min(1e-3)).max().item()
    out["packed"]["max_rel_err_vs_exact"] = rel
    # instruction-issue roofline: the exact kernel issues 2 FP32-pipe instructions
    # per term, the packed one 1 (two packed-half2 instructions per two terms)
    out["exact"]["frac_of_issue"] = 2 * terms / (out["exact"]["ms"] / 1e3) / issue_peak
    out["packed"]["frac_of_issue"] = 1 * terms / (out["packed"]["ms"] / 1e3) / issue_peak
    out["workload"] = "config2 forward, fp16 Q [32,2,3136,32], K^T [32,2,32,49]"
    out["issue_peak"] = "148 SMs x 128 lanes x sampled clock; exact: 2 FP32 instructions per term, packed: 1 per term"
    return out


def newton_section(dev, steps, warmup, flush, stream, peaks, peak_kind):
    """Configuration 3: 4096 SPD 128x128 matrices, 12 iterations, fp32:
    scaled-transpose init in split3 and mixed arithmetic, and the drop-in
    NewtonInverse_forward (reference init, A + 0.01 I, split3) that the
    reference arm times; matrices/s and the tensor-pipe roofline."""
    from laplacianformer_b200 import capi, workloads

    batch = 4096
    w = workloads.config3(device=dev, batch=batch)
    A, iters = w["A"], w["iters"]
    X = torch.empty_like(A)
    out = {}
    flops = batch * iters * 4.0 * 128 ** 3
    # products issued per iteration, in units of one 128^3 product: H = P V
    # (3 terms on full iterations) and Y = V G (2 terms on full iterations)
    runs = (("split3", capi.INIT_SCALED_TRANSPOSE, 0.0, capi.PREC_SPLIT3, 5.0),
            ("mixed", capi.INIT_SCALED_TRANSPOSE, 0.0, capi.PREC_MIXED, (5.0 * 2 + 2.0 * (iters - 2)) / iters),
            ("dropin", capi.INIT_REFERENCE, 0.01, capi.PREC_SPLIT3, 5.0))
    for name, init, reg, prec, units in runs:
        def step():
            capi.newton_inverse_fwd(A, iters, init_mode=init, reg=reg, precision=prec, out=X)
        times = time_steps(step, max(2, steps // 2), max(3, warmup), flush, stream)
        ms = max_over_ranks(statistics.mean(times))
        res = capi.newton_inverse_residual(A, X, reg)
        ach = flops / (ms / 1e3) / 1e12
        out[name] = {
            "value": batch / (ms / 1e3), "unit": "matrices/s", "ms_per_step": ms,
            "init": "reference (A + 0.01 I, alpha = 1.8/rowsum^2), the drop-in NewtonInverse_forward"
                    if name == "dropin" else "scaled transpose (A^T / (||A||_1 ||A||_inf))",
            "residual_fro_max": float(res.max().item()), "residual_fro_mean": float(res.mean().item()),
            "roofline": {"bound": "tensor", "kernel": "ns_tc_fwd_kernel", "achieved": ach,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": ach / peaks["bf16_tflops"],
                         "peak_kind": f"bf16 dense burst, {peak_kind} (kind::f16 MMAs run at the same rate)",
                         "algorithmic": "4*N^3 per matrix per iteration",
                         "issued_products_per_iteration": units,
                         "issued_tensor_tflops": units / 2.0 * ach,
                         "issued_frac": units / 2.0 * ach / peaks["bf16_tflops"],
                         "traffic": NCU_TRAFFIC["ns_tc_fwd_kernel"] if name == "split3" else None,
                         "algorithmic_bytes_per_launch": batch * 2 * 128 * 128 * 4},
        }
    return out


# DRAM bytes of one launch of each kernel, from the ncu captures summarised
# under profiles/ (dram__bytes_read.sum + dram__bytes_write.sum).
NCU_TRAFFIC = {"lsub_bwd_fast_kernel": 65.50e6 + 1.96e6, "lsub_fwd_kernel": 26.15e6 + 0.13e6,
               # the 4096-matrix configuration-3 launch, split3 (the written X partly still in L2 at exit)
               "ns_tc_fwd_kernel": 268.9e6 + 217.0e6}


def copy_bound_ms(hin, din, hout, dout, steps, dev):
    """Host<->device copies of one step alone: the inputs H2D on one stream and
    the outputs D2H on another (PCIe is full duplex), as the pipeline overlaps
    them; mean ms over `steps`."""
    s1, s2 = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    times = []
    for it in range(steps + 2):
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(s1)
        s2.wait_event(a)
        with torch.cuda.stream(s1):
            for h, d in zip(hin, din):
                d.copy_(h, non_blocking=True)
        with torch.cuda.stream(s2):
            for h, d in zip(hout, dout):
                h.copy_(d, non_blocking=True)
        s1.wait_stream(s2)
        b.record(s1)
        torch.cuda.synchronize()
        if it >= 2:
            times.append(a.elapsed_time(b))
    return statistics.mean(times)


def run_b200(args, rank, world, dev):
    # Clocks over every timed region of the run (the headline loop alone is a
    # few ms, shorter than one nvidia-smi sample period).
    with ClockSampler(dev.index) as clk_all:
        line = _run_b200(args, rank, world, dev)
    line["clocks_headline_loop"] = line.pop("clocks")
    line["clocks"] = clk_all.summary()
    line["clocks"]["scope"] = "sampled every 200 ms from before the first warm-up to after the last record"
    return line


def _run_b200(args, rank, world, dev):
    from laplacianformer_b200 import capi, workloads

    peaks, peak_kind = _peaks()
    stream = torch.cuda.current_stream(dev)
    flush = _flush_buffer(dev)
    dtype = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[args.dtype]
    w = workloads.config2(device=dev, dtype=dtype, seed=rank)
    q, kT, ds = w["q"], w["kT"], w["ds"]
    B, H, N, D = q.shape
    M = kT.shape[-1]
    bh = B * H
    s = torch.empty(B, H, N, M, device=dev, dtype=dtype)
    dq = torch.empty_like(q)
    dk = torch.empty_like(kT)
    ws_bytes = capi.laplace_sub_bwd_workspace_size(q, kT)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None

    ev_f = []
    ev_b = []

    def step():
        a = torch.cuda.Event(enable_timing=True)
        m_ = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        capi.laplace_sub_fwd(q, kT, s)
        m_.record(stream)
        capi.laplace_sub_bwd(ds, q, kT, dq, dk, workspace=ws)
        e.record(stream)
        ev_f.append((a, m_))
        ev_b.append((m_, e))

    with ClockSampler(dev.index) as clk:
        times = time_steps(step, args.steps, args.warmup, flush, stream)
    torch.cuda.synchronize()
    timed_f = ev_f[-args.steps:]
    timed_b = ev_b[-args.steps:]
    fwd_ms_r = statistics.mean(a.elapsed_time(b) for a, b in timed_f)
    bwd_ms_r = statistics.mean(a.elapsed_time(b) for a, b in timed_b)
    ms_r = statistics.mean(times)
    ranks = per_rank([ms_r, fwd_ms_r, bwd_ms_r])
    ms = max(r[0] for r in ranks)
    fwd_ms = max(r[1] for r in ranks)
    bwd_ms = max(r[2] for r in ranks)
    dists = bh * N * M  # per rank per step
    value = world * dists / (ms / 1e3) / 1e9

    es = q.element_size()
    fb, bb = laplace_bytes(bh, N, M, D, es)
    terms = bh * N * M * D
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    clock_mhz = clk.summary()["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
    issue_peak = sm_count * 4 * 32 * clock_mhz * 1e6  # FP32 lane-operations/s at the sampled clock
    bwd_ops = 4 * terms  # sub, step (fma.sat), two fma per term; packed f32x2 forms count as 2
    roofline = {
        "bound": "fp32_issue", "kernel": "lsub_bwd_fast_kernel balanced (fused dQ + dK^T) + lsub_bwd_dk_finalize",
        "achieved": bwd_ops / (bwd_ms / 1e3) / 1e12, "peak": issue_peak / 1e12, "unit": "T FP32 lane-ops/s",
        "frac": bwd_ops / (bwd_ms / 1e3) / issue_peak,
        "peak_kind": f"{sm_count} SMs x 128 FP32 lanes x {clock_mhz:.0f} MHz (median SM clock sampled in the timed region)",
        "algorithmic_ops_per_launch": bwd_ops,
        "ops_per_term": "4 FP32 lane-operations (sub, fma.sat step, 2 fma); the kernel issues them as 2.5 instructions "
                        "per term with packed f32x2 forms, each of which occupies the FP32 pipe for 2 lane-operations",
        "traffic": NCU_TRAFFIC["lsub_bwd_fast_kernel"] if dtype == torch.float32 else None,
        "algorithmic_bytes_per_launch": bb,
        "hbm": {"achieved_gbs": bb / (bwd_ms / 1e3) / 1e9, "peak_gbs": peaks["hbm_gbs"],
                "frac": bb / (bwd_ms / 1e3) / 1e9 / peaks["hbm_gbs"], "peak_kind": peak_kind},
        "fwd": {"ms": fwd_ms, "kernel": "lsub_fwd_kernel", "ops_per_term": 2,
                "frac": 2 * terms / (fwd_ms / 1e3) / issue_peak,
                "hbm_gbs": fb / (fwd_ms / 1e3) / 1e9,
                "traffic": NCU_TRAFFIC["lsub_fwd_kernel"] if dtype == torch.float32 else None},
        "step_frac": 6 * terms / (ms / 1e3) / issue_peak,
    }

    # End to end through the public API: pinned host buffers in, results out.
    hq = q.cpu().pin_memory()
    hk = kT.cpu().pin_memory()
    hg = ds.cpu().pin_memory()
    hs = torch.empty(s.shape, dtype=dtype).pin_memory()
    hdq = torch.empty(dq.shape, dtype=dtype).pin_memory()
    hdk = torch.empty(dk.shape, dtype=dtype).pin_memory()

    from laplacianformer_b200.streaming import HostPipeline

    pipe = HostPipeline(q.shape, M, dtype=dtype, device=dev, chunks=8)

    def e2e_step():
        pipe(hq, hk, hg, hs, hdq, hdk)

    e2e_times = time_steps(e2e_step, args.steps, args.warmup, flush, stream)
    e2e_ms = max_over_ranks(statistics.mean(e2e_times))
    copy_ms = max_over_ranks(copy_bound_ms((hq, hk, hg), (q, kT, ds), (hs, hdq, hdk), (s, dq, dk), 5, dev))
    h2d = (q.numel() + kT.numel() + ds.numel()) * es
    d2h = (s.numel() + dq.numel() + dk.numel()) * es

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": {"fp32": "f32", "fp16": "f16", "bf16": "bf16"}[args.dtype],
        "data": "synthetic (seeded N(0,1), configuration-2 shapes)",
        "config": {"workload": f"config2 LaplaceSub fwd+bwd {args.dtype}: Q [{B * world},{H},{N},{D}] "
                               f"(per rank [{B},{H},{N},{D}]), K^T [.,{H},{D},{M}], dS [.,{H},{N},{M}]",
                   "global_batch": B * world, "seq_len": N, "landmarks": M, "channels": D,
                   "parallelism": f"bh-shard x{world}, no collective",
                   "l2": "flushed between timed steps (256 MB write outside the events)"},
        "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
        "per_rank": {"fields": ["step_ms", "fwd_ms", "bwd_ms"], "values": ranks},
        "roofline": roofline,
        "e2e": {"value": world * dists / (e2e_ms / 1e3) / 1e9, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "copy_bound_ms": copy_ms, "frac_of_copy_bound": copy_ms / e2e_ms,
                "api": "laplacianformer_b200.streaming.HostPipeline (C ABI, 8 B*H chunks on copy-in / kernel / "
                       "copy-out streams) with pinned host buffers; copy_bound_ms = the same copies alone, both "
                       "PCIe directions overlapped"},
        "gpu_launches": (3 if ws is not None else 2) * args.steps,
        "clocks": clk.summary(),
    }
    if not args.skip_newton:
        line["newton_inverse"] = newton_section(dev, args.steps, args.warmup, flush, stream, peaks, peak_kind)
        line["gpu_launches"] += 3 * max(2, args.steps // 2)
    if not args.skip_config5:
        for key, ntok in (("config5", args.n_tokens), ("config5_long", args.n_tokens_long)):
            if ntok <= 0:
                continue
            c5 = config5_record(args, rank, world, dev, ntok, args.gather if world > 1 else "none", flush)
            line[key] = c5
            line["gpu_launches"] += c5.pop("launches")
            torch.cuda.empty_cache()
    if world == 1:
        line["packed_fp16"] = packed_fp16_record(dev, args.steps, args.warmup, flush, stream, issue_peak)
        line["gpu_launches"] += 2 * args.steps
    if world == 1 and not args.skip_config4:
        c4 = config4_record(args, dev, flush, stream)
        line["config4"] = c4
        line["gpu_launches"] += c4.pop("launches")
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_laplace({"q": q, "kT": kT, "ds": ds}, os.cpu_count() or 1)
        line["cpu_baseline_eager"] = cpu_baseline_eager({"q": q, "kT": kT, "ds": ds}, os.cpu_count() or 1)
    return line


def config5_record(args, rank, world, dev, n_tokens, gather, flush):
    """Configuration 5: B=8, H=16, D=64, M=256 chunk-mean landmarks, bf16 Q/K,
    LaplaceSub fwd+bwd plus the 256x256 landmark-kernel inverse (fp32, 10
    iterations).  Strong scaling: the 128 (b,h) slices are split over ranks,
    and dQ, dK^T and X end up replicated on every rank (S stays sharded:
    gathering it would move more bytes over NVLink than the sharded compute
    saves).  gather "peer": the backward stores every dQ tile into all ranks'
    IPC-mapped gather buffers as it computes it, dK^T and X are pushed by a
    put kernel, and a stream-ordered flag barrier ends the step; gather
    "after": the same outputs all-gathered over NCCL after the compute (also
    timed beside "peer" as the collective baseline, with the gather alone)."""
    from laplacianformer_b200 import capi, workloads
    from laplacianformer_b200.sharding import shard_bounds

    stream = torch.cuda.current_stream(dev)
    B, H, D, M, N = 8, 16, 64, 256, n_tokens
    lo, hi = shard_bounds(B * H, world, rank)
    bh = hi - lo
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    q = torch.randn(1, bh, N, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, bh, N, D, generator=g, device=dev).to(torch.bfloat16)
    L = workloads.chunk_mean_landmarks(k, M)
    kT = L.transpose(-1, -2).contiguous()
    ds = torch.randn(1, bh, N, M, generator=g, device=dev).to(torch.bfloat16)
    del k
    s = torch.empty(1, bh, N, M, device=dev, dtype=torch.bfloat16)
    Lf = L.float().contiguous()
    LfT = Lf.transpose(-1, -2).contiguous()
    A = torch.empty(1, bh, M, M, device=dev)
    ws = torch.empty(max(1, capi.laplace_sub_bwd_workspace_size(q, kT)), dtype=torch.uint8, device=dev)
    sigma = math.sqrt(D)
    chunk = -(-(B * H) // world)
    steps = max(3, min(args.steps, 10))

    side = torch.cuda.Stream(dev)

    def compute(dq, dk, X, dq_peers=None):
        # The landmark inverse does not depend on the distances: it runs on a
        # second stream beside them (its few 4-CTA clusters are latency-bound
        # and would otherwise leave most SMs idle at the end of the step).
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            capi.laplace_kernel_fwd(Lf, LfT, -1.0 / sigma, out=A)  # exp(-cdist_1 / sigma), S never stored
            capi.newton_inverse_fwd(A, 10, out=X)
        capi.laplace_sub_fwd(q, kT, s)
        if dq_peers:
            capi.laplace_sub_bwd_peers(ds, q, kT, dq, dk, dq_peers, workspace=ws)
        else:
            capi.laplace_sub_bwd(ds, q, kT, dq, dk, workspace=ws)
        stream.wait_stream(side)

    dq, dk = torch.empty_like(q), torch.empty_like(kT)
    X = torch.empty_like(A)
    rec = {}
    if gather in ("after", "peer"):
        # NCCL baseline: replicated dQ, dK^T and X through all_gather_into_tensor
        gbufs = [torch.empty((world * chunk,) + tuple(t.shape[2:]), device=dev, dtype=t.dtype) for t in (dq, dk, X)]
        sends = [t[0] if bh == chunk else torch.zeros((chunk,) + tuple(t.shape[2:]), device=dev, dtype=t.dtype)
                 for t in (dq, dk, X)]

        def gather_all():
            for i, (t, buf) in enumerate(zip((dq, dk, X), gbufs)):
                if bh != chunk:
                    sends[i][:bh].copy_(t[0])
                torch.distributed.all_gather_into_tensor(buf, sends[i] if bh != chunk else t[0])

        def step_after():
            compute(dq, dk, X)
            gather_all()

        t_after = statistics.mean(time_steps(step_after, steps, max(3, args.warmup), flush, stream))
        t_gather = statistics.mean(time_steps(gather_all, steps, 3, flush, stream))
        del gbufs, sends
        rec["nccl_after"] = [t_after, t_gather]
    if gather == "peer":
        from laplacianformer_b200.peer import PeerGather

        try:
            pg = PeerGather([((N, D), q.dtype), ((D, M), kT.dtype), ((M, M), torch.float32)], B * H, device=dev)
        except RuntimeError as exc:  # every rank raises together; report the NCCL variant instead
            rec["peer_error"] = str(exc)[:300]
            gather = "after"
    if gather == "peer":
        pdq, pdk, pX = (pg.local(i)[:bh].unsqueeze(0) for i in range(3))
        peers = [pg.peer_ptrs(i) for i in range(3)]

        def step():
            compute(pdq, pdk, pX, peers[0])
            capi.peer_put(pdk[0], peers[1])
            capi.peer_put(pX[0], peers[2])
            pg.barrier(stream)

        times = time_steps(step, steps, max(3, args.warmup), flush, stream)
        torch.cuda.synchronize(dev)
        status = capi.device_status(clear=True)
        if status != capi.LF_OK:
            raise RuntimeError(f"peer gather: device status {status} (a barrier wait expired)")
        pg.close()
        launches = steps * 8  # fwd, bwd + its dK finalize, landmark kernel, inverse, 2 puts, barrier
        parallelism = ("dQ stored into every rank's IPC-mapped gather buffer by the backward kernel itself, "
                       "dK^T/X pushed by a put kernel, flag barrier (no collective)")
    elif gather == "after":
        times = time_steps(step_after, steps, max(3, args.warmup), flush, stream) if "nccl_after" not in rec \
            else [rec["nccl_after"][0]] * steps
        launches = steps * 5  # NCCL's gathers are not ours
        parallelism = "dQ/dK^T/X all_gather_into_tensor over NCCL after the compute"
    else:
        times = time_steps(lambda: compute(dq, dk, X), steps, max(3, args.warmup), flush, stream)
        launches = steps * 5  # fwd, bwd + its dK finalize, landmark kernel, inverse
        parallelism = "no collective"
    after = rec.get("nccl_after", [0.0, 0.0])
    ranks = per_rank([statistics.mean(times), after[0], after[1]])
    ms = max(r[0] for r in ranks)
    out = {
        "value": B * H * N * M / (ms / 1e3) / 1e9, "unit": UNIT, "ms_per_step": ms, "steps": steps,
        "scaling": "strong", "dtype": "bf16 (inverse fp32)",
        "workload": f"config5 N={N}: LaplaceSub fwd+bwd bf16 (B*H=128, M=256, D=64) + NewtonInverse 256x256 fp32 x10",
        "parallelism": f"bh-shard x{world} (strong), " + parallelism,
        "newton_matrices_per_s": B * H / (ms / 1e3),
        "per_rank": {"fields": ["step_ms", "nccl_after_step_ms", "nccl_gather_only_ms"], "values": ranks},
        "l2": "inputs larger than L2" if N >= 16384 else "flushed between timed steps",
        "launches": launches,
    }
    if "peer_error" in rec:
        out["peer_error"] = rec["peer_error"]
    if "nccl_after" in rec:
        out["nccl_after_step_ms"] = max(r[1] for r in ranks)
        out["gather_ms"] = max(r[2] for r in ranks)
    else:
        out["gather_ms"] = 0.0
    return out


def config4_record(args, dev, flush, stream):
    """Configuration 4: the Laplacian attention block forward + backward, bf16
    Q/K/V [128,8,196,64], 49 landmarks from 2x2 pooling of K, 8 iterations."""
    from laplacianformer_b200 import workloads
    from laplacianformer_b200.attention import laplacian_attention, pool_landmarks

    w = workloads.config4(device=dev, batch=128)
    q, k, v = (w[x].detach().requires_grad_() for x in ("q", "k", "v"))
    up = torch.randn_like(q)

    def step():
        L = pool_landmarks(k, 14, 2)  # the landmarks carry K's gradient, as in the block
        out = laplacian_attention(q, k, v, L, iters=8, sigma=8.0)
        out.backward(up)

    steps = max(3, min(args.steps, 10))
    times = time_steps(step, steps, max(3, args.warmup), flush, stream)
    ms = statistics.mean(times)
    tokens = 128 * 196
    return {"value": tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "workload": "config4 Laplacian attention block fwd+bwd: Q,K,V [128,8,196,64] bf16, M=49 (2x2 pooling "
                        "of K inside the step, gradients through it), sigma=8, NewtonInverse 8 iterations; landmark "
                        "inverse fused (A built in-kernel); exp(-S/sigma) fused into the distance kernels both ways",
            "launches": steps * 9}


def run_config5(args, rank, world, dev):
    """--workload config5: the configuration-5 record as the line itself."""
    flush = _flush_buffer(dev)
    with ClockSampler(dev.index) as clk:
        rec = config5_record(args, rank, world, dev, args.n_tokens, args.gather if world > 1 else "none", flush)
    launches = rec.pop("launches")
    return {
        "metric": METRIC, "value": rec["value"], "unit": UNIT, "n_gpus": world, "steps": rec["steps"],
        "warmup": max(3, args.warmup), "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), configuration-5 shapes)",
        "config": {"workload": rec["workload"], "global_batch": 8, "heads": 16, "seq_len": args.n_tokens,
                   "parallelism": rec["parallelism"], "l2": rec["l2"]},
        "gather_ms": rec["gather_ms"], "per_rank": rec["per_rank"],
        **{k: rec[k] for k in ("nccl_after_step_ms", "peer_error") if k in rec},
        "newton_matrices_per_s": rec["newton_matrices_per_s"], "gpu_launches": launches, "clocks": clk.summary(),
    }


def run_reference(args, rank, world, dev):
    from oracle.build_ref import load_ref

    if args.workload == "config5":
        return {"impl": "reference", "unavailable": "configuration 5 needs bf16 LaplaceSubtraction (no bf16 dispatch, "
                "LaplaceSubtraction_cuda_kernel.cu:471), n = 256 NewtonInverse (rejected above 128, "
                "NewtonInverse_cuda_kernel.cu:726) and 64-bit offsets (int indexing overflows at N = 262144)"}
    ref = load_ref()
    if ref is None:
        return {"impl": "reference", "unavailable": "oracle/_ref/Laplace_subtraction_cuda_ref.so not built "
                "(python oracle/build_ref.py needs the reference sources)"}
    from laplacianformer_b200 import workloads

    stream = torch.cuda.current_stream(dev)
    flush = _flush_buffer(dev)
    dtype = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[args.dtype]
    if dtype == torch.bfloat16:
        return {"impl": "reference", "unavailable": "the reference LaplaceSubtraction has no bf16 dispatch "
                "(src/LaplaceSubtraction_cuda_kernel.cu:471)"}
    w = workloads.config2(device=dev, dtype=dtype, seed=rank)
    q, kT, ds = w["q"], w["kT"], w["ds"]
    B, H, N, D = q.shape
    M = kT.shape[-1]
    s = torch.empty(B, H, N, M, device=dev, dtype=dtype)
    dq = torch.empty_like(q)
    dk = torch.empty_like(kT)

    def step():
        ref.LaplaceSubtraction_forward(q, kT, s)
        ref.LaplaceSubtraction_backward_query(ds, q, kT, dq)
        ref.LaplaceSubtraction_backward_key(ds, q, kT, dk)

    with ClockSampler(dev.index) as clk:
        times = time_steps(step, args.steps, args.warmup, flush, stream)
    ms = statistics.mean(times)
    value = B * H * N * M / (ms / 1e3) / 1e9
    # The same end-to-end step as the B200 arm: pinned host inputs copied in,
    # the reference operators, results copied out.
    hq, hk, hg = q.cpu().pin_memory(), kT.cpu().pin_memory(), ds.cpu().pin_memory()
    hs = torch.empty(s.shape, dtype=dtype).pin_memory()
    hdq = torch.empty(dq.shape, dtype=dtype).pin_memory()
    hdk = torch.empty(dk.shape, dtype=dtype).pin_memory()

    def e2e_step():
        q.copy_(hq, non_blocking=True)
        kT.copy_(hk, non_blocking=True)
        ds.copy_(hg, non_blocking=True)
        step()
        hs.copy_(s, non_blocking=True)
        hdq.copy_(dq, non_blocking=True)
        hdk.copy_(dk, non_blocking=True)

    e2e_ms = statistics.mean(time_steps(e2e_step, args.steps, args.warmup, flush, stream))
    es = q.element_size()
    h2d = (q.numel() + kT.numel() + ds.numel()) * es
    d2h = (s.numel() + dq.numel() + dk.numel()) * es
    # Newton–Schulz on configuration 3 with the reference operator (its own init).
    from laplacianformer_b200 import workloads as W

    A = W.config3(device=dev, batch=4096)["A"]
    X = torch.empty_like(A)
    nt = time_steps(lambda: ref.NewtonInverse_forward(A, X, 12), max(2, args.steps // 2), max(3, args.warmup),
                    flush, stream)
    nms = statistics.mean(nt)
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": {"fp32": "f32", "fp16": "f16"}[args.dtype],
        "data": "synthetic (seeded N(0,1), configuration-2 shapes)",
        "config": {"workload": f"config2 LaplaceSub fwd+bwd {args.dtype}: Q [{B},{H},{N},{D}], K^T [{B},{H},{D},{M}]",
                   "global_batch": B, "seq_len": N, "parallelism": "single GPU (rank 0 only)",
                   "l2": "flushed between timed steps"},
        "device": "the reference's own CUDA operators (oracle/_ref, built from its sources for sm_100) on 1 B200",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": 0, "kind": "reference",
                         "sample": "full workload; the reference has no CPU implementation, its CUDA kernels run on the GPU"},
        "e2e": {"value": B * H * N * M / (e2e_ms / 1e3) / 1e9, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "the reference's Laplace_subtraction_cuda ops with pinned host buffers copied in and out"},
        "newton_inverse": {"value": 4096 / (nms / 1e3), "unit": "matrices/s", "ms_per_step": nms,
                           "init": "reference (A + 0.01 I, alpha = 1.8/rowsum^2)"},
        "clocks": clk.summary(),
    }


def run_only(args, dev):
    """One workload, no sampling or baselines (for ncu launch lists and captures)."""
    from laplacianformer_b200 import capi, workloads

    stream = torch.cuda.current_stream(dev)
    flush = _flush_buffer(dev)
    if args.only == "laplace":
        dtype = {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[args.dtype]
        w = workloads.config2(device=dev, dtype=dtype)
        q, kT, ds = w["q"], w["kT"], w["ds"]
        s = torch.empty(q.shape[0], q.shape[1], q.shape[2], kT.shape[3], device=dev, dtype=dtype)
        dq, dk = torch.empty_like(q), torch.empty_like(kT)
        ws_bytes = capi.laplace_sub_bwd_workspace_size(q, kT)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None

        def step():
            capi.laplace_sub_fwd(q, kT, s)
            capi.laplace_sub_bwd(ds, q, kT, dq, dk, workspace=ws)
    else:
        A = workloads.config3(device=dev, batch=args.ns_batch)["A"]
        X = torch.empty_like(A)

        def step():
            capi.newton_inverse_fwd(A, 12, init_mode=capi.INIT_SCALED_TRANSPOSE, out=X)
    times = time_steps(step, args.steps, args.warmup, flush, stream)
    print(json.dumps({"only": args.only, "ms_per_step": statistics.mean(times), "steps": args.steps}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--dtype", choices=["fp32", "fp16", "bf16"], default="fp32")
    ap.add_argument("--skip-newton", action="store_true")
    ap.add_argument("--only", choices=["laplace", "newton"], default=None,
                    help="profiling aid: run one workload only and print its timings")
    ap.add_argument("--ns-batch", type=int, default=4096)
    ap.add_argument("--workload", choices=["config2", "config5"], default="config2")
    ap.add_argument("--n-tokens", type=int, default=16384, help="configuration-5 sequence length")
    ap.add_argument("--n-tokens-long", type=int, default=65536,
                    help="sequence length of the second configuration-5 sub-record (0: leave it out)")
    ap.add_argument("--gather", choices=["none", "after", "peer"], default="peer",
                    help="config 5 with N>1: replicate dQ, dK^T and X on every rank by peer stores from the kernels "
                         "(peer; the NCCL variant is timed beside it), by NCCL after the compute (after), or not at all")
    ap.add_argument("--skip-config5", action="store_true", help="leave the configuration-5 sub-record out")
    ap.add_argument("--skip-config4", action="store_true", help="leave the configuration-4 sub-record out")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)

    if args.impl == "reference":
        if rank != 0:
            return
        line = run_reference(args, rank, world, dev)
        print(json.dumps(line), flush=True)
        return

    if args.only:
        run_only(args, dev)
        return
    if world > 1:
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        torch.distributed.init_process_group("nccl", device_id=dev)
    try:
        line = run_config5(args, rank, world, dev) if args.workload == "config5" else run_b200(args, rank, world, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if torch.distributed.is_initialized():
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
