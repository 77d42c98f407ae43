"""Benchmark of the fused diagonal-covariance EM iteration on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flashgmm|reference]
                    [--workload c2]

One *step* is one EM iteration (Pass 1 + Pass 2 statistics, stats allreduce when
N > 1, M-step update) over the workload's points, inputs resident in HBM.  The
metric is EM iterations/s of the named workload (default ``c2``: N=65,536,
K=256, d=128).  With --gpus N > 1 (launched under torch.distributed.run, one
rank per GPU, NCCL) every rank owns a full c2-sized shard of one larger data
set (weak scaling) and ``value`` counts c2-sized iterations completed by all
ranks per second.

Rank 0 prints ONE JSON line.  Besides the contract keys it carries ``roofline``
(dominant kernel, CUDA-event timed inside this run), ``cpu_baseline`` (the
reference's own C++/OpenMP op on this host's cores, N=1 only), ``e2e`` (whole
EM iterations through the public op with every step's inputs copied from pinned host
memory and its results read back), ``clocks`` (nvidia-smi
sampled during the timed region) and ``gpu_launches``.

``--impl reference`` times the reference's CPU implementation of the same step
(``oracle/_ref``, built from the reference sources; else the C restatement) on
the host cores, rank 0 only.
"""
import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from flashgmm_b200.data import WORKLOADS, make_workload  # noqa: E402

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


# --------------------------------------------------------------------------- utils
def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                "source": "fallback"}


def algorithmic(wl, n_points):
    """Per-iteration algorithmic work of one EM iteration (the survey's measurement row).

    FLOPs, in fp32-product units: each of the two contractions the design executes is
    2 N K (2 d) multiply-adds = 4 N K d (distance GEMM [x^2 | x] . [1/var | -2 mu/var],
    statistics GEMM gamma^T [x^2 | x]); 8 N K d per iteration (the reference's recompute
    design counts a third, 12 N K d, reported beside it).  Bytes: X read once, the
    log-normalizer written, the parameters read and written and the statistics written:
    4 (N d + N + 4 K d + 2 K), all fp32.  Whatever the design moves beyond that shows in
    the measured traffic, not here."""
    N, K, d = n_points, wl.K, wl.d
    flops = 8.0 * N * K * d
    nbytes = 4.0 * (N * d + N + 4 * K * d + 2 * K)
    return flops, nbytes


def ncu_traffic(kernel, workload):
    """DRAM bytes per launch (read + write) of `kernel` on `workload` from the committed
    ncu summary profiles/ncu_traffic.txt (lines: kernel workload bytes), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "ncu_traffic.txt")) as f:
            for ln in f:
                p = ln.split()
                if len(p) >= 3 and not ln.startswith("#") and p[0] == kernel and p[1] == workload:
                    return float(p[2])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.idx)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thr = threading.Thread(target=self._read, daemon=True)
            self.thr.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thr.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def gpu_id(dev):
    """nvidia-smi -i selector for a torch device (UUID: immune to CUDA_VISIBLE_DEVICES)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        return str(dev.index or 0)


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ------------------------------------------------------------------ reference arm
def load_reference_op():
    """The reference's own CPU op (oracle/_ref) or, if it is not built, the C restatement."""
    try:
        from oracle.build_ref import load_ref
        R = load_ref()
        return (lambda X, mu, var, lp: R.flash_em_fused(X, mu, var, lp, 64, 8)), "reference"
    except Exception:
        from oracle import oracle
        return (lambda X, mu, var, lp: [torch.from_numpy(a) for a in
                                        oracle.flash_em_fused(X, mu, var, lp, BK=8)]), "port"


def cpu_time_per_iter(wl, budget_s=12.0, min_iters=2):
    """Time the reference CPU op on a bounded sample of the workload.  Returns
    (seconds per full-size iteration, sample description, kind, threads)."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    op, kind = load_reference_op()
    # size the sample so one iteration takes ~budget/4
    n = min(wl.N, 4096)
    X, mu, var, lp = make_workload(wl, N=n)
    t0 = time.perf_counter()
    op(X, mu, var, lp)
    t1 = time.perf_counter() - t0
    per_point = t1 / n
    n = int(min(wl.N, max(1024, (budget_s / 4) / max(per_point, 1e-12))))
    X, mu, var, lp = make_workload(wl, N=n)
    its, t_tot = 0, 0.0
    while its < min_iters or t_tot < budget_s * 0.5:
        t0 = time.perf_counter()
        mu, var, lp, ln = op(X, mu, var, lp)
        t_tot += time.perf_counter() - t0
        its += 1
        if t_tot > budget_s:
            break
    s_iter_sample = t_tot / its
    s_iter_full = s_iter_sample * wl.N / n  # cost is exactly linear in N
    sample = (f"{its} iterations at N={n} of workload {wl.name} (K={wl.K}, d={wl.d}), "
              f"{s_iter_sample:.3f} s/iter, scaled x{wl.N / n:.2f} to N={wl.N}")
    return s_iter_full, sample, kind, threads


def run_reference(args, wl):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    op, kind = load_reference_op()
    # each step: one EM iteration; on a sample of the workload if the full size is slow
    n = min(wl.N, 4096)
    X, mu, var, lp = make_workload(wl, N=n)
    t0 = time.perf_counter()
    op(X, mu, var, lp)
    per_point = (time.perf_counter() - t0) / n
    budget_total = 150.0
    per_step = budget_total / max(1, args.steps + args.warmup)
    n = int(min(wl.N, max(1024, per_step / max(per_point, 1e-12))))
    X, mu, var, lp = make_workload(wl, N=n)
    for _ in range(args.warmup):
        mu, var, lp, ln = op(X, mu, var, lp)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        mu, var, lp, ln = op(X, mu, var, lp)
    dt = time.perf_counter() - t0
    s_iter = dt / args.steps * wl.N / n
    value = 1.0 / s_iter
    sample = (f"{args.steps} iterations at N={n} of workload {wl.name}, scaled x{wl.N / n:.2f} "
              f"to N={wl.N} (cost linear in N)")
    line = {
        "impl": "reference", "metric": f"EM iterations/s ({wl.name}: N={wl.N}, K={wl.K}, d={wl.d})",
        "value": value, "unit": "iter/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": s_iter * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": wl.name, "N": wl.N, "K": wl.K, "d": wl.d, "device": "host cpu"},
        "cpu_baseline": {"value": value, "unit": "iter/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": "iter/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------------ our arm
def profile_dominant(C, X, points, mu, var, lp, ws, reps=5):
    """CUDA-event durations of the launches of one em_stats call, summed per kernel name
    (a kernel runs once per point chunk), averaged over `reps` calls: ms per iteration."""
    import ctypes
    from flashgmm_b200 import _lib
    lib = _lib.load()
    N, d = X.shape
    K = mu.shape[0]
    nmax = 128  # the library times at most 128 launches of a call
    acc, seen = {}, {}
    for _ in range(reps):
        ms = (ctypes.c_float * nmax)()
        names = (ctypes.c_char_p * nmax)()
        _lib.check(lib.fgmm_em_stats_profiled(
            X.data_ptr(), points.data_ptr() if points is not None else None, N, d, mu.data_ptr(),
            var.data_ptr(), lp.data_ptr(), K, ws.stats.data_ptr(), ws.ln.data_ptr(),
            ws.ws.data_ptr(), ws.ws.numel(), torch.cuda.current_stream().cuda_stream, ms, names,
            nmax))
        for i in range(nmax):
            if names[i] is None:
                break
            acc[names[i].decode()] = acc.get(names[i].decode(), 0.0) + ms[i]
            seen[names[i].decode()] = seen.get(names[i].decode(), 0) + 1
    # With many point chunks not every launch is timed: scale each per-chunk kernel's sum by
    # (its launches per call) / (its timed launches per call).
    total = lib.fgmm_em_stats_launches(N, d, K)
    chunks = max(1, (total - 2) // 3)
    out = {}
    for k, v in acc.items():
        per_call = seen[k] / reps
        want = 1 if ("prep" in k or "reduce" in k) else chunks
        out[k] = v / reps * (want / per_call if per_call < want else 1.0)
    return out


def run_ours(args, wl):
    ws_n, rank, local = dist_env()
    if ws_n > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from flashgmm_b200 import _lib
    from flashgmm_b200 import flash_gmm_native as C
    lib = _lib.load()

    # each rank: a full workload-sized shard of an (n_gpus x N)-point data set
    n_total = wl.N * ws_n
    X, mu, var, lp = make_workload(wl, N=n_total, rows=(rank * wl.N, (rank + 1) * wl.N))
    X, mu0, var0, lp0 = (t.to(dev).contiguous() for t in (X, mu, var, lp))
    N, d, K = wl.N, wl.d, wl.K
    points = C.prepare_points(X, K)
    ws = C.StatsWorkspace(N, d, K, dev)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    mu, var, lp = mu0.clone(), var0.clone(), lp0.clone()

    prepared = [False]
    tc_family = C.family_for(N, d, K) == 2

    def step():
        nonlocal mu, var, lp
        if ws_n == 1:  # statistics and update in one call (update fused into the reduction;
            # it also builds the next step's parameter operands, so no separate preparation)
            C.em_step(X, mu, var, lp, points=points, workspace=ws, out=(mu, var, lp),
                      prepared=prepared[0])
            prepared[0] = tc_family
            return
        # statistics over this rank's shard (the parameter operands left by the previous
        # update), one all-reduce, the update that also prepares the next operands
        stats, _ = C.em_stats(X, mu, var, lp, points=points, workspace=ws, prepared=prepared[0])
        dist.all_reduce(stats)
        if tc_family:
            C.em_update_prepared(stats, n_total, points, ws, out=(mu, var, lp))
            prepared[0] = True
        else:
            mu, var, lp = C.em_update(stats, n_total, K, d)

    clocks = ClockSampler(gpu_id(dev)).start() if rank == 0 else None
    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    if ws_n > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()  # untimed: evict X / operands from L2 between iterations
        ev[i][0].record()
        step()
        ev[i][1].record()
    torch.cuda.synchronize()
    if ws_n > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    total_ms = sum(a.elapsed_time(b) for a, b in ev)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if ws_n > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = t.item()
    ms_per_step = total_ms / args.steps
    value = ws_n * 1000.0 / ms_per_step  # workload-sized iterations per second, all ranks

    # dominant kernel: per-launch CUDA-event durations of the em_stats sequence
    prof = profile_dominant(C, X, points, mu, var, lp, ws)
    dom = max(prof, key=prof.get)
    pk = peaks()
    f16x3 = pk["bf16_tflops"] / 3.0  # three fp16 products (kind::f16, bf16 rate) per fp32 product
    flops, nbytes = algorithmic(wl, N)
    gemm = dom in ("tc_pass1_kernel", "tc_stats_kernel")
    if gemm:  # each of the two kernels carries one of the two contractions
        achieved = flops / 2.0 / (prof[dom] * 1e-3) / 1e12
        roofline = {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": f16x3,
                    "unit": "TFLOP/s", "frac": achieved / f16x3}
    else:
        achieved = nbytes / (prof[dom] * 1e-3) / 1e9
        roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": pk["hbm_gbs"],
                    "unit": "GB/s", "frac": achieved / pk["hbm_gbs"]}
    roofline.update({
        "traffic": ncu_traffic(dom, wl.name), "kernel_ms": prof[dom], "launch_ms": prof,
        "peak_note": (f"3xF16 effective = {pk['source']} bf16 {pk['bf16_tflops']:.0f} TF/s / 3 "
                      f"(three fp16 products per fp32 product); hbm {pk['source']} "
                      f"{pk['hbm_gbs']:.0f} GB/s"),
        "iteration_frac": (flops / (ms_per_step * 1e-3) / 1e12) / f16x3,
        "iteration_frac_12nkd": (1.5 * flops / (ms_per_step * 1e-3) / 1e12) / f16x3,
        "traffic_over_algorithmic": None,  # set below
        "algorithmic": {"flops_per_iter": flops, "bytes_per_iter": nbytes,
                        "dominant_flops_per_launch": flops / 2.0 if gemm else None}})

    if roofline["traffic"]:
        roofline["traffic_over_algorithmic"] = roofline["traffic"] / nbytes

    # one EM step: em_stats' launches; on the tensor-core family less the parameter
    # preparation (the previous update wrote the operands), and on several GPUs plus the
    # separate update launch after the all-reduce
    launches = lib.fgmm_em_stats_launches(N, d, K) - (1 if tc_family else 0) + (1 if ws_n > 1 else 0)
    e2e = None
    cpu = None
    if not args.no_e2e:
        e2e = run_e2e(wl, dev, args, ws_n, rank)
    c5 = None
    if not args.no_strong_c5:
        t_n, t_1 = strong_c5(dev, ws_n, rank)
        if rank == 0:
            c5 = {"workload": "c5 (N=2^24, K=1024, d=128, points split over the GPUs)",
                  "ms_per_iter": t_n, "ms_per_iter_1gpu": t_1, "speedup": t_1 / t_n,
                  "iters": 10, "n_gpus": ws_n}
    if rank == 0 and ws_n == 1 and not args.no_cpu_baseline:
        s_full, sample, kind, threads = cpu_time_per_iter(wl)
        cpu = {"value": 1.0 / s_full, "unit": "iter/s", "cores": threads, "kind": kind,
               "sample": sample}
    if rank == 0:
        line = {
            "metric": f"EM iterations/s ({wl.name}: N={wl.N}, K={wl.K}, d={wl.d})",
            "value": value, "unit": "iter/s", "n_gpus": ws_n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl.name, "N_per_gpu": N, "K": K, "d": d,
                       "N_total": n_total, "parallelism": f"dp{ws_n}" if ws_n > 1 else "single",
                       "family": {1: "simt", 2: "tcgen05", 3: "lowk"}.get(C.family_for(N, d, K), "?"),
                       "l2": "flushed between timed iterations (256 MB write, untimed)"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": launches * args.steps, "strong_c5": c5,
        }
        print(json.dumps(line), flush=True)
    if ws_n > 1:
        dist.destroy_process_group()


def strong_c5(dev, ws_n, rank, iters=10, warmup=2):
    """Strong scaling on configuration 5 (N = 2^24 unit-norm points, K = 1024, d = 128): the
    points are split evenly over the ranks and every iteration all-reduces the statistics.
    Returns (ms per iteration, max over ranks; ms per iteration of the whole set on rank 0's
    GPU alone, measured in the same run).  The points are generated on the GPUs (the same
    distribution as the workload generator: noisy unit directions, renormalised)."""
    from flashgmm_b200 import flash_gmm_native as C
    Ntot, K, d = 1 << 24, 1024, 128
    g = torch.Generator().manual_seed(5)
    u = torch.randn(K, d, generator=g)
    u = u / u.norm(dim=1, keepdim=True)
    mu0 = (u + 0.05 * torch.randn(K, d, generator=g))
    mu0 = (mu0 / mu0.norm(dim=1, keepdim=True)).to(dev)
    var0 = torch.ones(K, d, device=dev)
    lp0 = torch.full((K,), -math.log(K), device=dev)
    ud = u.to(dev)

    def shard(n, seed):
        gg = torch.Generator(device=dev).manual_seed(seed)
        z = torch.randint(0, K, (n,), generator=gg, device=dev)
        x = ud[z] + 0.05 * torch.randn(n, d, generator=gg, device=dev)
        return (x / x.norm(dim=1, keepdim=True)).contiguous()

    def run(X, n_total, group_size):
        pts = C.prepare_points(X, K)
        ws = C.StatsWorkspace(X.shape[0], d, K, dev)
        mu, var, lp = mu0.clone(), var0.clone(), lp0.clone()
        prepared = False
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for it in range(warmup + iters):
            if it == warmup:
                torch.cuda.synchronize(dev)
                if group_size > 1:
                    dist.barrier()
                e0.record()
            stats, _ = C.em_stats(X, mu, var, lp, points=pts, workspace=ws, prepared=prepared)
            if group_size > 1:
                dist.all_reduce(stats)
            C.em_update_prepared(stats, n_total, pts, ws, out=(mu, var, lp))
            prepared = True
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / iters

    one = None
    if rank == 0:  # the whole set on one GPU, for the speed-up
        X = shard(Ntot, 1234)
        one = run(X, Ntot, 1)
        del X
        torch.cuda.empty_cache()
    if ws_n > 1:
        dist.barrier()
        X = shard(Ntot // ws_n, 1000 + rank)
        t = torch.tensor([run(X, Ntot, ws_n)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        many = t.item()
        del X
    else:
        many = one
    return many, one


def run_e2e(wl, dev, args, ws_n=1, rank=0, steps=200):
    """The same metric through the public API from HOST buffers.  Every step copies this
    rank's X shard and the current parameters from pinned host memory to the GPU, runs one
    EM iteration (``flash_gmm_native.flash_em_fused`` on one GPU; ``em_stats`` +
    ``all_reduce`` + ``em_update`` on several) and reads the new parameters and the log
    normaliser back into pinned host memory.  The X copy of step i + 1 runs on a second
    stream into a second device buffer while step i computes.  Wall clock over `steps`
    steps after a warm-up, max over ranks; value counts workload-sized iterations of all
    ranks per second."""
    from flashgmm_b200 import flash_gmm_native as C
    n_total = wl.N * ws_n
    X, mu, var, lp = make_workload(wl, N=n_total, rows=(rank * wl.N, (rank + 1) * wl.N))
    Xh = X.pin_memory()
    ph = [t.pin_memory() for t in (mu, var, lp)]
    N, d, K = wl.N, wl.d, wl.K
    Xd = [torch.empty_like(X, device=dev) for _ in range(2)]
    pd = [[torch.empty_like(t, device=dev) for t in ph] for _ in range(2)]
    out_h = [torch.empty_like(t).pin_memory() for t in ph] + [torch.empty(N).pin_memory()]
    copy = torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)
    landed = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]
    ws = C.StatsWorkspace(N, d, K, dev) if ws_n > 1 else None

    def issue_copy(i):
        # all host-to-device traffic of step i on the copy stream (a small copy queued on
        # the compute stream would wait behind the next step's X copy in the copy engine)
        b = i % 2
        with torch.cuda.stream(copy):
            copy.wait_event(freed[b])
            for t, h in zip(pd[b], ph):
                t.copy_(h, non_blocking=True)
            Xd[b].copy_(Xh, non_blocking=True)
            landed[b].record(copy)

    def step(i):
        b = i % 2
        comp.wait_event(landed[b])
        mu_d, var_d, lp_d = pd[b]
        if ws_n > 1:
            stats, ln = C.em_stats(Xd[b], mu_d, var_d, lp_d, workspace=ws)
            dist.all_reduce(stats)
            out = list(C.em_update(stats, n_total, K, d)) + [ln]
        else:
            out = C.flash_em_fused(Xd[b], mu_d, var_d, lp_d)
        freed[b].record(comp)
        for h, t in zip(out_h, out):
            h.copy_(t, non_blocking=True)

    def run(n):
        issue_copy(0)
        for i in range(n):
            if i + 1 < n:
                issue_copy(i + 1)
            step(i)
        torch.cuda.synchronize(dev)

    run(3)
    if ws_n > 1:
        dist.barrier()
    t0 = time.perf_counter()
    run(steps)
    dt = (time.perf_counter() - t0) / steps
    if ws_n > 1:
        t = torch.tensor([dt], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = t.item()
    h2d = Xh.numel() * 4 + sum(t.numel() * 4 for t in ph)
    d2h = sum(t.numel() * 4 for t in out_h)
    # the copy-only bound: this rank's X shard over PCIe from pinned memory, timed alone
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    Xd[0].copy_(Xh, non_blocking=True)
    e0.record()
    for _ in range(5):
        Xd[0].copy_(Xh, non_blocking=True)
    e1.record()
    torch.cuda.synchronize(dev)
    h2d_gbs = 5 * Xh.numel() * 4 / (e0.elapsed_time(e1) * 1e-3) / 1e9
    return {"value": ws_n / dt, "unit": "iter/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "h2d_gbs": h2d_gbs,
            "copy_bound_iter_s": ws_n * h2d_gbs * 1e9 / h2d,
            "step": ("H2D of X and the parameters from pinned host memory, one EM iteration "
                     "through flashgmm_b200.flash_gmm_native, D2H of the new parameters and "
                     "log-normalizer; X copies double-buffered on a second stream (per-rank "
                     "bytes)")}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="flashgmm", choices=["flashgmm", "reference"])
    ap.add_argument("--workload", default="c2", choices=sorted(WORKLOADS))
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-strong-c5", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
