"""Benchmark of the attention + matmul2d hot path on B200 (one process per GPU).

Metric: "attention & matmul2d TFLOP/s (% of B200 peak)".  One step = the two BASELINE configs
the north star targets, sharded across the N ranks with no data-path collective:
  * config 3: causal bf16 attention, Q/K/V [B=8, H=16, S=2048, D=128] -> 128 (b,h) units,
    units/N per rank; algorithmic FLOPs 4*S^2*D/2 per unit (causal half) = 1.074 GFLOP.
  * config 4: bf16 GEMM 8192^3 (fp32 accumulate, bf16 out) -> A row-blocks of 8192/N rows per
    rank, B replicated; FLOPs 2*M*N*K = 1.0995 TFLOP in total.
value = total algorithmic FLOPs of the step / step time (max over ranks), TFLOP/s, strong
scaling (the total work is the config; ranks split it).  Within a step the GEMM runs on the
launching stream and the attention on a second stream started with it (the two are independent;
attention CTAs fill the SMs that the GEMM's last round of tiles leaves idle); `parts` gives the
GEMM's duration inside the step and the attention's alone from a separate sequential pass.  The assembling all-gather of the
outputs (the library's lcCommAllGatherRows: NCCL over NVLink, overlapped with the GEMM) is timed
separately and reported under `assemble`.

Inputs are synthetic (seeded normal / uniform as BASELINE.json describes), larger than L2 for the
GEMM; L2 is flushed (a 256 MiB write) between timed steps.  Kernel times are CUDA events on the
launching stream.  `e2e` runs the same step through the C ABI with host (pinned) buffers and the
reference's default IO policy (upload, download, synchronize), copies included.

--impl reference times the reference's own CPU implementation (oracle/_ref, built from the
reference sources) on a bounded sample of the same workload on the host cores.
"""
import argparse
import ctypes as C
import json
import os
import sys
import time

import numpy as np

_JSON_FD = 1


def emit(line: dict) -> None:
    os.write(_JSON_FD, (json.dumps(line) + "\n").encode())

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "lightining-core_b200", "python"))

B, H, S, D = 8, 16, 2048, 128
UNITS = B * H
GM = GN = GK = 8192
ATTN_FLOPS_PER_UNIT = 4.0 * S * S * D / 2.0  # causal: half the S x S tile work (FA convention)
GEMM_FLOPS = 2.0 * GM * GN * GK
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name> ('traffic_bytes_per_launch:')."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class Clocks:
    """SM clock and throttle reasons sampled during the timed region.

    Polls NVML every 10 ms from a thread (reading only; nothing is set), so even a short timed
    region gets samples.  Without NVML the summary says "no samples"."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = set()
        self.smax = None
        self._stop = None
        self._thread = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.smax = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - sampling is best effort
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for name, bit in self.REASONS.items():
                        if mask & bit:
                            self.reasons.add(name)
                except Exception:  # noqa: BLE001
                    pass
                self._stop.wait(0.01)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *a):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.smax, "samples": 0, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.smax, "samples": len(self.samples),
                "reasons": sorted(self.reasons), "source": "NVML, 10 ms polling during the timed steps"}


# ----------------------------------------------------------------------------- reference arm
def cpu_sample(threads, heads=32, rows=256):
    """Reference CPU path on a bounded sample of the workload: `heads` causal attention units and
    `rows` rows of the 8192^3 GEMM.  Returns (TFLOP/s, seconds, sample description)."""
    from oracle import oracle as O

    kind = "reference" if O.ref_available() else "port"
    L = O.ref() if kind == "reference" else O.port()
    rng = np.random.default_rng(2)
    bfr = O.port().bf16_round
    q, k, v = (bfr(rng.standard_normal((heads, S, D), dtype=np.float32)) for _ in range(3))
    a = bfr((rng.uniform(-1, 1, (rows, GK)) / np.sqrt(GK)).astype(np.float32))
    bm = bfr((rng.uniform(-1, 1, (GK, GN)) / np.sqrt(GK)).astype(np.float32))
    t0 = time.perf_counter()
    L.attention_units(q, k, v, causal=True, threads=threads)
    t1 = time.perf_counter()
    L.matmul(a, bm, threads=threads)
    t2 = time.perf_counter()
    flops = heads * ATTN_FLOPS_PER_UNIT + 2.0 * rows * GN * GK
    desc = (f"{heads} of 128 causal heads [2048,128] + {rows} of 8192 GEMM rows (8192x8192), bf16-rounded "
            f"inputs widened to fp32; attention {t1 - t0:.2f}s, gemm {t2 - t1:.2f}s on {threads} threads")
    return flops / (t2 - t0) / 1e12, t2 - t0, desc, kind


def run_reference(args, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    vals = []
    for i in range(args.warmup + args.steps):
        v, secs, desc, kind = cpu_sample(threads)
        if i >= args.warmup:
            vals.append((v, secs))
    val = float(np.median([x[0] for x in vals]))
    ms = float(np.median([x[1] for x in vals])) * 1e3
    line = {"metric": "attention & matmul2d TFLOP/s (% of B200 peak)", "value": val, "unit": "TFLOP/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": dict(CONFIG, parallelism=f"cpu threads x{threads} (bounded sample of the workload)"),
            "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": desc},
            "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


CONFIG = {"workload": "cfg3 causal attention bf16 [8,16,2048,128] + cfg4 matmul2d bf16 8192^3 (fp32 accumulate)",
          "attention": "B=8 H=16 S=2048 D=128 causal, N(0,1) bf16, scale 1/sqrt(128)",
          "gemm": "M=N=K=8192, U(-1,1)/sqrt(K) bf16, row-major, bf16 out",
          "l2": "flushed between timed steps (256 MiB write); GEMM inputs 268 MB > L2"}


# ----------------------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import lightning_core_b200 as lc

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    L = lc.lib

    # ---- shards: units [u0, u1) of attention, rows [r0, r1) of the GEMM
    u0, u1 = lc.shard_range(UNITS, rank, world)
    r0, r1 = lc.shard_range(GM, rank, world)
    nu, nr = u1 - u0, r1 - r0

    g = torch.Generator(device=dev)
    g.manual_seed(2)
    qkv = torch.randn((3, UNITS, S, D), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    q, k, v = (qkv[i, u0:u1].contiguous() for i in range(3))
    del qkv
    attn_out = torch.empty_like(q)
    g.manual_seed(3)
    A = ((torch.rand((GM, GK), generator=g, device=dev) * 2 - 1) / GK ** 0.5).to(torch.bfloat16)[r0:r1].contiguous()
    Bm = ((torch.rand((GK, GN), generator=g, device=dev) * 2 - 1) / GK ** 0.5).to(torch.bfloat16)
    Cm = torch.empty((nr, GN), device=dev, dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, device=dev, dtype=torch.uint8)
    torch.cuda.synchronize()

    side = torch.cuda.Stream()
    sp_side = C.c_void_p(side.cuda_stream)

    def attn(stream_ptr=sp):
        lc.check(L.lcAttentionForward(C.c_void_p(q.data_ptr()), C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                                      C.c_void_p(attn_out.data_ptr()), nu, S, D, 1, lc.BF16, None, stream_ptr),
                 "attention")

    def gemm():
        lc.check(L.lcMatMul(C.c_void_p(A.data_ptr()), C.c_void_p(Bm.data_ptr()), C.c_void_p(Cm.data_ptr()), nr, GK,
                            GN, lc.BF16, None, sp), "matmul")

    def f32gemm_fn():
        # Strict fp32 matmul 2048^3 (config 2 family) through the default dispatch (3xTF32).
        n = 2048
        g.manual_seed(1)
        fa = torch.rand((n, n), generator=g, device=dev) * 2 - 1
        fb = torch.rand((n, n), generator=g, device=dev) * 2 - 1
        fc = torch.empty_like(fa)
        return lambda: lc.check(L.lcMatMul(C.c_void_p(fa.data_ptr()), C.c_void_p(fb.data_ptr()),
                                           C.c_void_p(fc.data_ptr()), n, n, n, lc.F32, None, sp), "matmul f32")

    def f32attn_fn():
        # Strict fp32 attention at the config-5 shape ([32, 3136, 64], non-causal), 3xTF32 path.
        g.manual_seed(4)
        fq, fk, fv = (torch.randn((32, 3136, 64), generator=g, device=dev) for _ in range(3))
        fo = torch.empty_like(fq)
        return lambda: lc.check(L.lcAttentionForward(C.c_void_p(fq.data_ptr()), C.c_void_p(fk.data_ptr()),
                                                     C.c_void_p(fv.data_ptr()), C.c_void_p(fo.data_ptr()), 32, 3136,
                                                     64, 0, lc.F32, None, sp), "attention f32")

    def cfg5_fn():
        # The integrated conv -> QKV -> attention -> projection pipeline at the config-5 shape.
        g.manual_seed(4)
        x = torch.randn((32, 64, 56, 56), generator=g, device=dev)
        w = (torch.rand((192, 64, 3, 3), generator=g, device=dev) * 2 - 1) * (6 / 576) ** 0.5
        bias = torch.zeros(192, device=dev)
        pw = (torch.rand((64, 64), generator=g, device=dev) * 2 - 1) * (6 / 64) ** 0.5
        out = torch.empty((32, 3136, 64), device=dev)
        return lambda: lc.check(L.lcConvAttentionNchw(C.c_void_p(x.data_ptr()), C.c_void_p(w.data_ptr()),
                                                      C.c_void_p(bias.data_ptr()), C.c_void_p(pw.data_ptr()),
                                                      C.c_void_p(out.data_ptr()), 32, 64, 56, 56, 192, 3, 3, 1, 1,
                                                      1, 1, 3136, 64, 64, 1, None, sp), "conv attention")

    if args.only:
        fn = {"gemm": gemm, "attention": attn, "f32gemm": None, "f32attn": None, "cfg5": None}[args.only]
        if fn is None:
            fn = {"f32gemm": f32gemm_fn, "f32attn": f32attn_fn, "cfg5": cfg5_fn}[args.only]()
        for _ in range(args.warmup + args.steps):
            fn()
        torch.cuda.synchronize()
        return

    for _ in range(args.warmup):
        attn()
        gemm()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    # The attention alone (sequential pass after the warm-up, same inputs, L2 flushed).
    attn_ms = []
    for i in range(min(args.steps, 10)):
        flush.zero_()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        attn()
        a1.record(stream)
        torch.cuda.synchronize()
        attn_ms.append(a0.elapsed_time(a1))
    # A step: the GEMM of this rank's rows on the launching stream and the attention of its units
    # on a second stream started with it (independent work: attention CTAs take the SMs the
    # GEMM's last round of tiles leaves idle), joined before the step's end event.  The GEMM's own
    # duration (events around it on its stream) carries the roofline; the attention's alone is
    # timed in the sequential pass above.
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    joined = [torch.cuda.Event() for _ in range(args.steps)]
    with Clocks(local_rank) as clk:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            side.wait_event(ev[i][0])
            gemm()
            ev[i][1].record(stream)
            attn(sp_side)
            joined[i].record(side)
            stream.wait_event(joined[i])
            ev[i][2].record(stream)
        torch.cuda.synchronize()
    clocks = clk.summary()
    gemm_ms = [e[0].elapsed_time(e[1]) for e in ev]
    step_ms = sum(e[0].elapsed_time(e[2]) for e in ev) / args.steps
    t = torch.tensor([step_ms, float(np.mean(attn_ms)), float(np.mean(gemm_ms))], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    step_ms, attn_avg, gemm_avg = (float(x) for x in t.tolist())
    total_flops = UNITS * ATTN_FLOPS_PER_UNIT + GEMM_FLOPS
    value = total_flops / (step_ms * 1e-3) / 1e12

    # ---- compute + assembling all-gather through the library's communicator: the attention
    # output's all-gather (NCCL over NVLink, side stream) overlaps the GEMM; then C is gathered.
    gather = None
    comm = None
    if world > 1:
        comm = make_comm(lc, torch, dist, rank, world, dev)
        gather = gathered_step(args, lc, torch, dist, comm, q, k, v, A, Bm, nu, nr, u0, r0, world, dev)

    # ---- e2e through the C ABI with host buffers and the reference's default policy
    e2e = e2e_run(args, lc, torch, q, k, v, A, Bm, nu, nr, world, dev, comm)

    # ---- extra configs: at N=1 the fp32 configs 1, 2, 5 and the HBM-bound ops; at N>1 config 5
    # sharded by image (its natural shard unit), the others being replicas-only sizes.
    if world == 1:
        extras = extra_configs(args, lc, torch, dev, sp)
    else:
        try:
            extras = sharded_cfg5(lc, torch, dev, sp, rank, world, comm)
        except Exception as exc:  # reported, never allowed to cost the headline line
            extras = {"cfg5_conv_attention_f32_sharded": {"error": f"{type(exc).__name__}: {exc}"}}

    if comm is not None:
        torch.cuda.synchronize()
        comm.close()
    if rank != 0:
        return
    pk, pk_kind = peaks()
    peak = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    gemm_ach = 2.0 * nr * GN * GK / (gemm_avg * 1e-3) / 1e12
    attn_ach = nu * ATTN_FLOPS_PER_UNIT / (attn_avg * 1e-3) / 1e12
    traffic = profile_traffic("gemm_bf16_8192.md")
    cpu = None
    if world == 1:
        cv, secs, desc, kind = cpu_sample(os.cpu_count() or 1)
        cpu = {"value": cv, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": kind, "sample": desc}
        # The reference itself is single-threaded: the same code on one host thread, smaller sample.
        cv1, _, desc1, _ = cpu_sample(1, heads=8, rows=64)
        cpu["single_thread"] = {"value": cv1, "unit": "TFLOP/s", "cores": 1, "sample": desc1}
    line = {
        "metric": "attention & matmul2d TFLOP/s (% of B200 peak)", "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": dict(CONFIG, parallelism=f"shard x{world}: attention units/{world}, gemm rows/{world}"),
        "frac_of_peak": value / peak, "peak_tflops": peak, "peak_kind": pk_kind,
        "parts": {"attention_ms": attn_avg, "attention_tflops": attn_ach, "attention_frac": attn_ach / peak,
                  "gemm_ms": gemm_avg, "gemm_tflops": gemm_ach, "gemm_frac": gemm_ach / peak,
                  "step_overlap_ms": attn_avg + gemm_avg - step_ms,
                  "how": "GEMM inside the timed step (attention on a second stream beside it); attention "
                         "alone in a sequential pass"},
        "roofline": {"bound": "tensor", "kernel": "gemm_bf16_tc2_kernel", "achieved": gemm_ach, "peak": peak,
                     "unit": "TFLOP/s", "frac": gemm_ach / peak,
                     "peak_source": f"{pk_kind} bf16_tflops (burst; kernel timed alone)",
                     "traffic": None if traffic is None else traffic * nr / GM},
        "assemble": gather,
        "e2e": e2e,
        "gpu_launches": 2 * args.steps * world,
        "clocks": clocks,
        "cpu_baseline": cpu,
        "extras": extras,
    }
    emit(line)


def make_comm(lc, torch, dist, rank, world, dev):
    """The library's NCCL communicator; rank 0's unique id travels over the torch process group."""

    def exchange(uid):
        t = torch.tensor(list(uid), dtype=torch.uint8, device=dev)
        dist.broadcast(t, 0)
        return bytes(t.cpu().tolist())

    return lc.Comm(rank, world, exchange)


def gathered_step(args, lc, torch, dist, comm, q, k, v, A, Bm, nu, nr, u0, r0, world, dev):
    """The step with its outputs assembled on every rank: attention of this rank's units, its
    all-gather (lcCommAllGatherRows: NCCL over NVLink) on a side stream overlapping the GEMM of
    this rank's rows, then the all-gather of C.  CUDA events on the launching stream, max over
    ranks; the all-gathers alone are timed too."""
    L = lc.lib
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    s = torch.cuda.current_stream()
    s2 = torch.cuda.Stream()
    sp, sp2 = C.c_void_p(s.cuda_stream), C.c_void_p(s2.cuda_stream)
    full_attn = torch.empty((UNITS, S, D), device=dev, dtype=torch.bfloat16)
    full_c = torch.empty((GM, GN), device=dev, dtype=torch.bfloat16)
    attn_rows, c_rows = full_attn[u0:u0 + nu], full_c[r0:r0 + nr]
    flush = torch.empty(256 << 20, device=dev, dtype=torch.uint8)

    def gathers(stream_ptr):
        lc.check(L.lcCommAllGatherRows(comm.handle, ptr(full_attn), UNITS, S * D * 2, stream_ptr), "gather attn")
        lc.check(L.lcCommAllGatherRows(comm.handle, ptr(full_c), GM, GN * 2, stream_ptr), "gather C")

    def step():
        lc.check(L.lcAttentionForward(ptr(q), ptr(k), ptr(v), ptr(attn_rows), nu, S, D, 1, lc.BF16, None, sp))
        e1 = torch.cuda.Event()
        e1.record(s)
        s2.wait_event(e1)
        lc.check(L.lcCommAllGatherRows(comm.handle, ptr(full_attn), UNITS, S * D * 2, sp2), "gather attn")
        lc.check(L.lcMatMul(ptr(A), ptr(Bm), ptr(c_rows), nr, GK, GN, lc.BF16, None, sp))
        e2 = torch.cuda.Event()
        e2.record(s)
        s2.wait_event(e2)
        lc.check(L.lcCommAllGatherRows(comm.handle, ptr(full_c), GM, GN * 2, sp2), "gather C")
        e3 = torch.cuda.Event()
        e3.record(s2)
        s.wait_event(e3)

    def timed(fn, reps):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        tot = 0.0
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            fn()
            e1.record(s)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        t = torch.tensor([tot / reps], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    reps = max(5, min(args.steps, 20))
    step_ms = timed(step, reps)
    gather_ms = timed(lambda: gathers(sp), reps)
    # the assembled outputs hold this rank's own rows where they belong
    ok = bool(torch.equal(full_attn[u0:u0 + nu], attn_rows)) and bool(torch.equal(full_c[r0:r0 + nr], c_rows))
    total_flops = UNITS * ATTN_FLOPS_PER_UNIT + GEMM_FLOPS
    out_bytes = (full_attn.numel() + full_c.numel()) * 2
    return {"ms_per_step": step_ms, "value": total_flops / (step_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "gather_only_ms": gather_ms, "bytes_assembled": out_bytes,
            "gather_recv_gbs_per_gpu": out_bytes * (world - 1) / world / (gather_ms * 1e-3) / 1e9,
            "own_rows_in_place": ok,
            "how": "attention -> all-gather (side stream) || GEMM -> all-gather, lcCommAllGatherRows (NCCL, "
                   "NVLink); CUDA events on the launching stream, L2 flushed between steps, max over ranks"}


def e2e_run(args, lc, torch, q, k, v, A, Bm, nu, nr, world, dev, comm=None):
    """Same step through the public C ABI with pinned host buffers: the reference's default IO
    policy (upload inputs, download output, synchronize) on each call, copies inside the timing.
    At N>1 the sharded entry points run it: each rank uploads its own units / rows and a 1/N slice
    of B (all-gathered over NVLink), and downloads its own output rows."""
    import torch.distributed as dist

    L = lc.lib
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    apol = lc.default_attention_policy()
    mpol = lc.default_matmul_policy()
    if comm is None:
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        ha, hb = A.cpu().pin_memory(), Bm.cpu().pin_memory()
        ho = torch.empty_like(hq).pin_memory()
        hc = torch.empty((nr, GN), dtype=torch.bfloat16).pin_memory()

        def step():
            lc.check(L.lcAttentionForward(ptr(hq), ptr(hk), ptr(hv), ptr(ho), nu, S, D, 1, lc.BF16, C.byref(apol),
                                          None), "attention e2e")
            lc.check(L.lcMatMul(ptr(ha), ptr(hb), ptr(hc), nr, GK, GN, lc.BF16, C.byref(mpol), None), "matmul e2e")
        h2d = (hq.numel() * 3 + ha.numel() + hb.numel()) * 2
        d2h = (ho.numel() + hc.numel()) * 2
    else:
        u0, _ = lc.shard_range(UNITS, comm.rank, world)
        r0, _ = lc.shard_range(GM, comm.rank, world)
        k0, k1 = lc.shard_range(GK, comm.rank, world)
        # Full-size pinned host arrays (the API describes the whole problem); each rank fills and
        # touches only its own part.
        hq, hk, hv = (torch.empty((UNITS, S, D), dtype=torch.bfloat16).pin_memory() for _ in range(3))
        for h, t in ((hq, q), (hk, k), (hv, v)):
            h[u0:u0 + nu].copy_(t.cpu())
        ha = torch.empty((GM, GK), dtype=torch.bfloat16).pin_memory()
        ha[r0:r0 + nr].copy_(A.cpu())
        hb = torch.empty((GK, GN), dtype=torch.bfloat16).pin_memory()
        hb[k0:k1].copy_(Bm[k0:k1].cpu())
        ho = torch.empty((UNITS, S, D), dtype=torch.bfloat16).pin_memory()
        hc = torch.empty((GM, GN), dtype=torch.bfloat16).pin_memory()

        def step():
            lc.check(L.lcAttentionForwardSharded(comm.handle, ptr(hq), ptr(hk), ptr(hv), ptr(ho), UNITS, S, D, 1,
                                                 lc.BF16, C.byref(apol), None), "attention e2e sharded")
            lc.check(L.lcMatMulSharded(comm.handle, ptr(ha), ptr(hb), ptr(hc), GM, GK, GN, lc.BF16, C.byref(mpol),
                                       None), "matmul e2e sharded")
        # bytes crossing PCIe on this rank, summed over ranks below
        h2d = (3 * nu * S * D + nr * GK + (k1 - k0) * GN) * 2
        d2h = (nu * S * D + nr * GN) * 2

    steps = max(2, min(args.steps, 5))
    for _ in range(2):
        step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = (time.perf_counter() - t0) / steps
    t = torch.tensor([dt, h2d, d2h], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t[:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[1:], op=dist.ReduceOp.SUM)
    dt, h2d, d2h = (float(x) for x in t.tolist())
    total_flops = UNITS * ATTN_FLOPS_PER_UNIT + GEMM_FLOPS
    return {"value": total_flops / dt / 1e12, "unit": "TFLOP/s", "ms_per_step": dt * 1e3,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "timing": "wall clock around synchronous C-ABI calls, max over ranks",
            "entry_points": "lcAttentionForward + lcMatMul" if comm is None else
            "lcAttentionForwardSharded + lcMatMulSharded (B: 1/N slice per rank over PCIe, all-gathered "
            "over NVLink; each rank downloads its own rows)", "steps": steps}


def sharded_cfg5(lc, torch, dev, sp, rank, world, comm):
    """Config 5 (conv [32,64,56,56] -> QKV -> attention -> projection, fp32) with the 32 images split
    across ranks by lcConvAttentionNchwSharded: compute + all-gather of [32, 3136, 64] on every rank,
    CUDA events, max over ranks."""
    import torch.distributed as dist

    L = lc.lib
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    stream = torch.cuda.current_stream()
    images = 32
    g = torch.Generator(device=dev)
    g.manual_seed(4)
    x = torch.randn((images, 64, 56, 56), generator=g, device=dev)
    bound = (6 / 576) ** 0.5
    w = (torch.rand((192, 64, 3, 3), generator=g, device=dev) * 2 - 1) * bound
    bias = torch.zeros(192, device=dev)
    g.manual_seed(5)
    pw = (torch.rand((64, 64), generator=g, device=dev) * 2 - 1) * (6 / 64) ** 0.5
    out = torch.empty((images, 3136, 64), device=dev)

    def run():
        lc.check(L.lcConvAttentionNchwSharded(comm.handle, ptr(x), ptr(w), ptr(bias), ptr(pw), ptr(out), images, 64,
                                              56, 56, 192, 3, 3, 1, 1, 1, 1, 3136, 64, 64, None, sp))

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    dist.barrier()
    reps = 5
    e0, e1 = (torch.cuda.Event(enable_timing=True) for _ in range(2))
    e0.record(stream)
    for _ in range(reps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    flops = 2 * 32 * 3136 * 192 * 576 + 32 * 4 * 3136 ** 2 * 64 + 2 * 32 * 3136 * 64 * 64
    return {"cfg5_conv_attention_f32_sharded": {"ms_with_gather": ms, "tflops": flops / (ms * 1e-3) / 1e12,
                                                "images_per_rank": f"{images}/{world}",
                                                "timing": "CUDA events, max over ranks; includes the all-gather"}}


def extra_configs(args, lc, torch, dev, sp):
    """The fp32 configs at N=1: attention [256,64] (cfg 1), matmul 1024^3 (cfg 2), the integrated
    conv->attention->projection pipeline [32,64,56,56] (cfg 5).  Device pointers, CUDA events."""
    L = lc.lib
    stream = torch.cuda.current_stream()
    ptr = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    g = torch.Generator(device=dev)
    res = {}

    def timeit(fn, reps):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps

    g.manual_seed(0)
    q, k, v = (torch.randn((256, 64), generator=g, device=dev) for _ in range(3))
    o = torch.empty_like(q)
    ms = timeit(lambda: lc.check(L.lcAttentionForward(ptr(q), ptr(k), ptr(v), ptr(o), 1, 256, 64, 0, lc.F32, None,
                                                      sp)), 50)
    res["cfg1_attention_f32_256x64"] = {"ms": ms, "tflops": 4 * 256 * 256 * 64 / (ms * 1e-3) / 1e12}
    for n in (256, 512, 1024, 2048):
        g.manual_seed(1)
        a = torch.rand((n, n), generator=g, device=dev) * 2 - 1
        b = torch.rand((n, n), generator=g, device=dev) * 2 - 1
        c = torch.empty_like(a)
        ms = timeit(lambda: lc.check(L.lcMatMul(ptr(a), ptr(b), ptr(c), n, n, n, lc.F32, None, sp)), 10)
        res[f"cfg2_matmul_f32_{n}"] = {"ms": ms, "tflops": 2 * n ** 3 / (ms * 1e-3) / 1e12}
    g.manual_seed(4)
    x = torch.randn((32, 64, 56, 56), generator=g, device=dev)
    bound = (6 / 576) ** 0.5
    w = (torch.rand((192, 64, 3, 3), generator=g, device=dev) * 2 - 1) * bound
    bias = torch.zeros(192, device=dev)
    g.manual_seed(5)
    pw = (torch.rand((64, 64), generator=g, device=dev) * 2 - 1) * (6 / 64) ** 0.5
    out = torch.empty((32, 3136, 64), device=dev)
    ms = timeit(lambda: lc.check(L.lcConvAttentionNchw(ptr(x), ptr(w), ptr(bias), ptr(pw), ptr(out), 32, 64, 56, 56,
                                                       192, 3, 3, 1, 1, 1, 1, 3136, 64, 64, 1, None, sp)), 3)
    flops = 2 * 32 * 3136 * 192 * 576 + 32 * 4 * 3136 ** 2 * 64 + 2 * 32 * 3136 * 64 * 64
    res["cfg5_conv_attention_f32"] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12}
    del x, out
    # HBM-bound elementwise ops against the measured copy bandwidth (inputs >> L2).
    pk, pk_kind = peaks()
    hbm = float(pk.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    n = 1 << 28
    va, vb = torch.rand(n, device=dev), torch.rand(n, device=dev)
    vc = torch.empty_like(va)
    ms = timeit(lambda: lc.check(L.lcVectorAdd(ptr(va), ptr(vb), ptr(vc), n, lc.F32, None, sp)), 10)
    gbs = 12.0 * n / (ms * 1e-3) / 1e9
    res["vector_add_f32_2^28"] = {"ms": ms, "gbs": gbs, "frac_of_hbm": gbs / hbm, "hbm_peak": f"{hbm} ({pk_kind})"}
    del va, vb, vc
    # fp32 configs against both nominal ceilings (no measured fp32 / tf32 peak is available):
    # CUDA-core fp32 = 148 SMs x 128 FMA/clk x 2 x 1.965 GHz; 3xTF32 = dense tf32 1125 / 3.
    for key in [k for k in res if k.startswith(("cfg1", "cfg2", "cfg5"))]:
        res[key]["frac_fp32_simt_nominal"] = res[key]["tflops"] / 74.4
        res[key]["frac_3xtf32_nominal"] = res[key]["tflops"] / 375.0
    # Config 4's GEMM sweep (bf16 in/out, fp32 accumulate), each size through lcMatMul's default
    # dispatch, L2 flushed before every timed launch (CUDA events on the launching stream).
    bf_peak = float(pk.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for (m, k, n) in ((16384, 1024, 4096), (4096, 4096, 4096), (16384, 16384, 16384)):
        g.manual_seed(3)
        a = ((torch.rand((m, k), generator=g, device=dev) * 2 - 1) / k ** 0.5).to(torch.bfloat16)
        b = ((torch.rand((k, n), generator=g, device=dev) * 2 - 1) / k ** 0.5).to(torch.bfloat16)
        c = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
        run = lambda: lc.check(L.lcMatMul(ptr(a), ptr(b), ptr(c), m, k, n, lc.BF16, None, sp))  # noqa: E731
        for _ in range(3):
            run()
        times = []
        for _ in range(5):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = sorted(times)[len(times) // 2]
        tf = 2.0 * m * k * n / (ms * 1e-3) / 1e12
        res[f"cfg4_matmul_bf16_{m}x{k}x{n}"] = {"ms": ms, "tflops": tf, "frac_of_bf16_peak": tf / bf_peak,
                                                "timing": "median of 5, L2 flushed before each"}
        del a, b, c
    del flush
    # Attention train step (forward + MSE loss + dV + SGD on V), fp32, 16 heads [1024, 64]:
    # forward 4*S^2*D plus dV = P^T dO 2*S^2*D per head (the P recomputation is not counted).
    g.manual_seed(6)
    tu, ts_, td = 16, 1024, 64
    tq, tk, tv, tt = (torch.randn((tu, ts_, td), generator=g, device=dev) for _ in range(4))
    to = torch.empty_like(tq)
    ms = timeit(lambda: lc.check(L.lcAttentionTrainStep(ptr(tq), ptr(tk), ptr(tv), ptr(tt), ptr(to), C.c_float(1e-3),
                                                        tu, ts_, td, 0, None, None, sp)), 10)
    tfl = 6.0 * ts_ * ts_ * td * tu / (ms * 1e-3) / 1e12
    res["train_step_f32_16x1024x64"] = {"ms": ms, "tflops": tfl, "frac_fp32_simt_nominal": tfl / 74.4}
    del tq, tk, tv, tt, to
    rows, cols = 65536, 1024
    x = torch.randn((rows, cols), device=dev)
    y = torch.empty_like(x)
    ms = timeit(lambda: lc.check(L.lcLayerNorm(ptr(x), ptr(y), rows, cols, 1e-5, sp)), 10)
    gbs = 8.0 * rows * cols / (ms * 1e-3) / 1e9
    res["layer_norm_f32_65536x1024"] = {"ms": ms, "gbs": gbs, "frac_of_hbm": gbs / hbm}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--only", default=None, choices=["gemm", "attention", "f32gemm", "f32attn", "cfg5"],
                    help="run only this kernel's warm-up + timed launches (for ncu captures); prints no JSON")
    args = ap.parse_args()
    # Libraries (NCCL's version banner, ...) may write to fd 1; keep it for the one JSON line only.
    global _JSON_FD
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist

        # NCCL's init lines (transport per channel: P2P/NVLS/...) go to stderr for the record.
        os.environ["NCCL_DEBUG"] = "INFO"
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT,GRAPH,NVLS")
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
