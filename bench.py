"""Benchmark: LaplaceSubtraction forward+backward (Gdist/s) on the pyramid-ViT
stage-1 shape, with the batched NewtonInverse (matrices/s) reported beside it.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

One process per GPU (torchrun for N > 1).  The path shards over B*H with no
collective: every rank runs its own batch-32 slice of a global batch 32*N
(weak scaling).  A step is one pass of the hot path over one batch: S =
LaplaceSub(Q, K^T), then both gradients (dQ, dK^T) of an upstream dS, through
the C ABI with inputs resident in HBM.  Timing: W untimed steps, then K steps
bracketed by a barrier and cudaDeviceSynchronize; each step is timed with CUDA
events on the launching stream and an L2 flush (a 256 MB write, outside the
events) separates steps; the max over ranks is reported.  rank 0 prints one
JSON line.

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


def time_steps(step, steps, warmup, flush, stream, kernel_events=None):
    """Warm up, then time `steps` calls of step() with events on `stream`."""
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs = []
    for _ in range(steps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        step()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    if torch.distributed.is_initialized():
        torch.distributed.barrier()
    return [a.elapsed_time(b) for a, b in evs]


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


def newton_section(dev, steps, warmup, flush, stream, peaks, peak_kind, quick=False):
    """Configuration 3: 4096 SPD 128x128 matrices, 12 iterations, fp32,
    scaled-transpose init; matrices/s and the tensor-pipe roofline."""
    from laplacianformer_b200 import capi, workloads

    batch = 4096
    w = workloads.config3(device=dev, batch=batch)
    A, iters = w["A"], w["iters"]
    X = torch.empty_like(A)
    out = {}
    for name, prec in (("split3", capi.PREC_SPLIT3), ("mixed", capi.PREC_MIXED)):
        def step():
            capi.newton_inverse_fwd(A, iters, init_mode=capi.INIT_SCALED_TRANSPOSE, precision=prec, out=X)
        times = time_steps(step, max(2, steps // 2), max(3, warmup), flush, stream)
        ms = max_over_ranks(statistics.mean(times))
        res = capi.newton_inverse_residual(A, X, 0.0)
        flops = batch * iters * 4.0 * 128 ** 3
        nmma = 3 if prec == capi.PREC_SPLIT3 else (3 * 2 + 1 * (iters - 2)) / iters
        out[name] = {
            "value": batch / (ms / 1e3), "unit": "matrices/s", "ms_per_step": ms,
            "residual_fro_max": float(res.max().item()), "residual_fro_mean": float(res.mean().item()),
            "roofline": {"bound": "tensor", "achieved": flops / (ms / 1e3) / 1e12,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                         "peak_kind": f"bf16 dense burst, {peak_kind} (kind::f16 MMAs run at the same rate)",
                         "algorithmic": "4*N^3 per matrix per iteration",
                         "issued_tensor_tflops": nmma * flops / (ms / 1e3) / 1e12,
                         "traffic": None},
        }
    return out


def run_b200(args, rank, world, dev):
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
    fwd_ms = statistics.mean(a.elapsed_time(b) for a, b in timed_f)
    bwd_ms = statistics.mean(a.elapsed_time(b) for a, b in timed_b)
    ms = max_over_ranks(statistics.mean(times))
    fwd_ms = max_over_ranks(fwd_ms)
    bwd_ms = max_over_ranks(bwd_ms)
    dists = bh * N * M  # per rank per step
    value = world * dists / (ms / 1e3) / 1e9

    es = q.element_size()
    fb, bb = laplace_bytes(bh, N, M, D, es)
    terms = bh * N * M * D
    sm_count = torch.cuda.get_device_properties(dev).multi_processor_count
    clock_mhz = clk.summary()["sm_mhz"] or peaks.get("sm_max_mhz", 1965.0)
    issue_peak = sm_count * 4 * 32 * clock_mhz * 1e6  # thread-instructions/s at the sampled clock
    roofline = {
        "bound": "hbm", "kernel": "lsub_bwd_fast_kernel balanced (fused dQ + dK^T) + lsub_bwd_dk_finalize",
        "achieved": bb / (bwd_ms / 1e3) / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
        "frac": bb / (bwd_ms / 1e3) / 1e9 / peaks["hbm_gbs"], "traffic": None,
        "peak_kind": peak_kind,
        "algorithmic_bytes_per_launch": bb,
        "note": "the kernel is bounded by the FP32 issue rate, not HBM; see 'issue'",
        "issue": {
            "instr_per_term": 4, "achieved_tinstr_s": 4 * terms / (bwd_ms / 1e3) / 1e12,
            "peak_tinstr_s": issue_peak / 1e12,
            "frac": 4 * terms / (bwd_ms / 1e3) / issue_peak,
            "peak_basis": f"{sm_count} SMs x 128 lanes x {clock_mhz:.0f} MHz (median sampled SM clock)",
        },
        "fwd": {"ms": fwd_ms, "achieved_gbs": fb / (fwd_ms / 1e3) / 1e9,
                "issue_frac": 2 * terms / (fwd_ms / 1e3) / issue_peak},
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
        "roofline": roofline,
        "e2e": {"value": world * dists / (e2e_ms / 1e3) / 1e9, "unit": UNIT, "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "api": "laplacianformer_b200.streaming.HostPipeline (C ABI, 8 B*H chunks on copy-in / kernel / copy-out streams) with pinned host buffers"},
        "gpu_launches": (3 if ws is not None else 2) * args.steps,
        "clocks": clk.summary(),
    }
    if not args.skip_newton:
        line["newton_inverse"] = newton_section(dev, args.steps, args.warmup, flush, stream, peaks, peak_kind)
        line["gpu_launches"] += sum(max(2, args.steps // 2) for _ in range(2))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_laplace({"q": q, "kT": kT, "ds": ds}, os.cpu_count() or 1)
    return line


def run_config5(args, rank, world, dev):
    """Configuration 5: B=8, H=16, D=64, M=256 chunk-mean landmarks, bf16 Q/K,
    LaplaceSub fwd+bwd plus the 256x256 landmark-kernel inverse (fp32, 10
    iterations).  Strong scaling: the 128 (b,h) slices are split over ranks."""
    from laplacianformer_b200 import capi, workloads
    from laplacianformer_b200.sharding import shard_bounds

    stream = torch.cuda.current_stream(dev)
    flush = _flush_buffer(dev)
    B, H, D, M, N = 8, 16, 64, 256, args.n_tokens
    lo, hi = shard_bounds(B * H, world, rank)
    bh = hi - lo
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    q = torch.randn(1, bh, N, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(1, bh, N, D, generator=g, device=dev).to(torch.bfloat16)
    L = workloads.chunk_mean_landmarks(k, M)
    kT = L.transpose(-1, -2).contiguous()
    ds = torch.randn(1, bh, N, M, generator=g, device=dev).to(torch.bfloat16)
    s = torch.empty(1, bh, N, M, device=dev, dtype=torch.bfloat16)
    dq, dk = torch.empty_like(q), torch.empty_like(kT)
    Lf = L.float().contiguous()
    LfT = Lf.transpose(-1, -2).contiguous()
    sll = torch.empty(1, bh, M, M, device=dev)
    X = torch.empty_like(sll)
    sigma = math.sqrt(D)

    gather = args.gather if world > 1 else "none"
    gbufs = None
    if gather != "none":
        # replicated dQ, dK^T and X on every rank (S stays sharded: gathering
        # it would move more bytes over NVLink than the sharded compute saves)
        gbufs = [torch.empty((world,) + tuple(t.shape), device=dev, dtype=t.dtype) for t in (dq, dk, X)]
    pieces = 4 if gather == "overlap" else 1
    per = -(-bh // pieces)
    bounds = [(i * per, min(bh, (i + 1) * per)) for i in range(pieces)]
    pbufs = []
    if gather == "overlap":  # one receive buffer per piece and output
        pbufs = [[torch.empty((world, b - a) + tuple(t.shape[2:]), device=dev, dtype=t.dtype) for t in (dq, dk, X)]
                 for a, b in bounds]

    def distances(a, b):
        sl = slice(a, b)
        capi.laplace_sub_fwd(q[:, sl], kT[:, sl], s[:, sl])
        capi.laplace_sub_bwd(ds[:, sl], q[:, sl], kT[:, sl], dq[:, sl], dk[:, sl])

    def inverse():
        capi.laplace_sub_fwd(Lf, LfT, sll)
        A = torch.exp(sll * (-1.0 / sigma))
        capi.newton_inverse_fwd(A, 10, out=X)

    def step():
        if gather == "none":
            distances(0, bh)
            inverse()
            return
        works = []
        for i, (a, b) in enumerate(bounds):
            distances(a, b)
            if gather == "overlap":  # piece i's dQ/dK^T cross NVLink while piece i+1 (and the inverse) compute
                for t, buf in zip((dq, dk), pbufs[i][:2]):
                    works.append(torch.distributed.all_gather_into_tensor(buf, t[0, a:b], async_op=True))
        inverse()
        if gather == "overlap":
            works.append(torch.distributed.all_gather_into_tensor(gbufs[2], X, async_op=True))
        if gather == "after":
            for t, buf in zip((dq, dk, X), gbufs):
                torch.distributed.all_gather_into_tensor(buf, t)
        for w in works:
            w.wait()

    times = time_steps(step, args.steps, args.warmup, flush, stream)
    ms = max_over_ranks(statistics.mean(times))
    return {
        "metric": METRIC, "value": B * H * N * M / (ms / 1e3) / 1e9, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), configuration-5 shapes)",
        "config": {"workload": f"config5 N={N}: LaplaceSub fwd+bwd bf16 (M=256, D=64) + NewtonInverse 256x256 fp32 x10",
                   "global_batch": B, "heads": H, "seq_len": N, "parallelism": f"bh-shard x{world} (strong), " + ("no collective" if gather == "none" else
                                   f"dQ/dK/X all-gathered ({gather})"),
                   "l2": "inputs larger than L2" if N >= 16384 else "flushed between timed steps"},
        "newton_matrices_per_s": B * H / (ms / 1e3),
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
    ap.add_argument("--gather", choices=["none", "after", "overlap"], default="none",
                    help="configuration 5 with N>1: all-gather dQ, dK^T and X after the compute or overlapped per piece")
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
