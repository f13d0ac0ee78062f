#!/usr/bin/env python
"""bench.py — the headline benchmark: (x)(+) pairs/s of mlu + lmul! on BASELINE config 2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--no-cpu-baseline] [--once]

Workload (config 2, the configuration the metric is quoted on that fits one GPU): mlu(MinPlus(), A) then
lmul!(F, B) in Float64 on a 256 x 256 4-connected grid digraph (65,536 vertices, 261,120 arcs with independent
weights uniform in [1, 10)); B is 65,536 x 256, Inf except 0.0 at 256 seeded distinct vertices, one per column.
Inputs are seeded synthetic data of exactly that shape (no dataset is involved).  A step is one pass of the hot
path: assembly of A into the factor (copyto!), the multifrontal factorization (lu!), and the solve.

  value  device-resident throughput: the weights and B already in HBM; per step the weights are re-assembled
         on the device (pp_update_values), factorized (pp_factor), B is reset from a device copy and solved in
         place (pp_lmul on device memory).  Timed with CUDA events on the library's stream over exactly K
         steps, bracketed by a barrier and a synchronize; max over ranks.
  e2e    the same metric through the C ABI with host buffers: pp_update_values from the host weights (H2D
         inside), pp_factor, pp_lmul on a pinned host B (H2D and D2H inside); host wall clock per step, summed.
  pairs  algorithmic: the partial LU of every front, sum_f sum_{t=na}^{nj-1} t^2, plus lmul!'s L* on the root
         paths of the 256 unit sources and U* over every front for all 256 columns (unpadded structure).

Multi-GPU (--gpus N under torchrun): one job on all ranks (strong scaling).  Every rank builds the same matrix;
the factorization is split (each rank factors its part of the bottom of the tree, NCCL broadcasts on the
library's stream give every rank the other parts, every rank factors the top), and each rank solves its own
column panel of B (256 / N columns); value = the job's pairs (the factorization once, every column's solve) /
the slowest rank's time.

--impl reference runs the reference's CPU algorithm (the oracle: the C restatement of PATHPACK.jl's CPU path,
oracle/; Julia is not available here) on the host cores, on the same workload; rank 0 only.

The default line also carries "mstar": config 4's mstar (mlu + Matrix(F), F32 MinPlus, directed 6-NN graph of
32,768 points, 4.3 GB of output) with its columns split into one contiguous panel per rank: wall seconds per
mstar at N GPUs (strong scaling; the factorization split as above, then one column panel of A* per rank).

--workload selects another BASELINE configuration instead, printing one line of the same form:
  config1, config3, config4   mlu + the whole star Matrix(F) as column panels over the ranks (device output;
                              e2e writes the panels into pinned host memory); cpu_baseline on a column sample
  config5a                    pp_getrf_batched over 4,096 128x128 MinPlus Int32 blocks
  config5b-i32/-f32/-f64      pp_gemm 8192^3: MinPlus Int32, MinPlus Float32, PlusProd Float64
"""
import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "pathpack.jl_b200"))
sys.path.insert(0, REPO)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


def ncu_traffic(path, kernel):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum, averaged over the captured launches)
    of the kernel in an ncu raw CSV export (`ncu -i <rep> --page raw --csv`) given with --traffic-csv, or None
    when no export is given."""
    if not path or not os.path.exists(path):
        return None
    import csv

    rows = list(csv.reader(open(path)))
    if len(rows) < 3:
        return None
    head = rows[0]
    try:
        kn, rd, wr = head.index("Kernel Name"), head.index("dram__bytes_read.sum"), head.index("dram__bytes_write.sum")
    except ValueError:
        return None
    unit = rows[1]
    scale = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}
    vals = []
    for r in rows[2:]:
        if len(r) > max(kn, rd, wr) and kernel.split("(")[0] in r[kn]:
            f = lambda i: float(r[i].replace(",", "")) * scale.get(unit[i], 1.0)
            vals.append(f(rd) + f(wr))
    return float(np.mean(vals)) if vals else None


# ----------------------------------------------------------------------------------------------- workloads

def config2(rank):
    from pathpack_b200 import graphs, ssymbolic

    n, I, J, W = graphs.grid2d(256, 256, 1.0, 10.0, seed=1000 + rank, dtype=np.float64)
    cp, rv, nz = graphs.csc(n, I, J, W)
    S = ssymbolic(n, cp, rv)
    k = 256
    B, src = graphs.unit_columns(n, k, seed=2000 + rank, dtype=np.float64)
    nn, na = S.nn.astype(np.float64), S.na.astype(np.float64)
    u_full = float((nn * (nn - 1) / 2 + nn * na).sum())
    pairs_solve = S.rootpath_pairs(S.invp[src]) + k * u_full
    return dict(name="mlu(MinPlus)+lmul! F64, 256x256 grid digraph (n=65536), B 65536x256 unit columns",
                semiring="MinPlus", dtype=np.float64, n=n, cp=cp, rv=rv, nz=nz, S=S, B=B, k=k,
                pairs_factor=S.pairs_factor(), pairs_solve=pairs_solve)


# star workloads (configs 1, 3, 4): mlu, then Matrix(F) as column panels; every rank builds the same matrix
# (the same seed) and computes its own contiguous block of columns of A*, kept in its GPU's memory
STAR = {
    "config1": dict(semiring="MinPlus", dtype=np.float64, cpu_cols=4096,
                    name="mstar(MinPlus) F64, 64x64 grid digraph (n=4096), 4096^2 output",
                    graph=lambda g: g.grid2d(64, 64, 1.0, 10.0, seed=11, dtype=np.float64)),
    "config3": dict(semiring="MaxMin", dtype=np.float32, cpu_cols=256,
                    name="mlu(MaxMin)+Matrix(F) F32, 40x40x40 7-point grid digraph (n=64000), 64000^2 output",
                    graph=lambda g: g.grid3d(40, 40, 40, seed=12, dtype=np.float32)),
    "config4": dict(semiring="MinPlus", dtype=np.float32, cpu_cols=2048,
                    name="mstar(MinPlus) F32, directed 6-NN of 32768 points (n=32768), 32768^2 output",
                    graph=lambda g: g.knn_directed(32768, 6, seed=13, dtype=np.float32)),
}


def star_workload(key):
    from pathpack_b200 import graphs, ssymbolic

    w = dict(STAR[key])
    n, I, J, W = w["graph"](graphs)
    cp, rv, nz = graphs.csc(n, I, J, W)
    t0 = time.perf_counter()
    S = ssymbolic(n, cp, rv)
    w.update(n=n, cp=cp, rv=rv, nz=nz, S=S, symbolic_s=time.perf_counter() - t0, pairs_factor=S.pairs_factor())
    nn, na = S.nn.astype(np.float64), S.na.astype(np.float64)
    w["per_column"] = float((nn * (nn - 1) / 2 + nn * na).sum())
    return w


def star_pairs(w, col0, ncols):
    """Algorithmic pairs of columns col0 .. col0+ncols-1 of A* = U* (L* I): L* on each source's root path, U*
    over every front for every column (unpadded structure)."""
    S = w["S"]
    return ncols * w["per_column"] + S.rootpath_pairs(S.invp[col0:col0 + ncols])


def alu_peak(semiring, dtype, sms, mhz):
    """Nominal ALU issue peak in (x)(+) pairs/s: SMs x SM clock x lanes per SM (128 for 32-bit, 64 for Float64)
    / the fewest instructions per pair on sm_100a (FADD2 + 3-input FMNMX: 1 for Float32 MinPlus/MaxPlus; a
    2-input min plus half a 3-input max: 1.5 for MaxMin/MinMax; add + min: 2 for Int32 and Float64; one fused
    multiply-add: 1 for PlusProd; one LOP3: 1 for OrAnd)."""
    dt = np.dtype(dtype)
    lanes = 64 if dt == np.float64 else 128
    if semiring in ("PlusProd", "OrAnd", "MaxProd"):
        c = 1.0
    elif dt == np.float64 or dt == np.int32:
        c = 2.0
    elif semiring in ("MaxMin", "MinMax"):
        c = 1.5
    else:
        c = 1.0
    return sms * mhz * 1e6 * lanes / c


# ----------------------------------------------------------------------------------------------- clocks

class Clocks:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.p, self.path = index, None, None

    def __enter__(self):
        try:
            self.path = "/tmp/pp_clocks_%d_%d.csv" % (os.getpid(), self.index)
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", "--query-gpu=" + self.Q, "--format=csv,noheader,nounits",
                                       "-i", str(self.index), "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
            # a timed region of a few tens of ms fits between two samples: start timing once the sampler runs, so
            # that at least the sample taken right after the warm-up (clocks under load) is recorded
            t0 = time.time()
            while time.time() - t0 < 3.0 and os.path.getsize(self.path) == 0:
                time.sleep(0.01)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
            self.f.close()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = [r.split(",") for r in open(self.path).read().strip().splitlines() if r.count(",") >= 8]
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------------------------- arms

def cpu_baseline(w, threads):
    """The oracle (the C restatement of the reference CPU path) on the full workload, timed on this host."""
    from oracle.oracle import OracleLU

    t0 = time.perf_counter()
    O = OracleLU(w["semiring"], w["dtype"], w["S"]).assemble(w["cp"], w["rv"], w["nz"]).factor(threads)
    X = O.lmul(w["B"], threads)
    dt = time.perf_counter() - t0
    return dt, X


def run_reference(args, rank, world):
    if rank != 0:
        return
    w = config2(0)
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        cpu_baseline(w, threads)
    tot = 0.0
    for _ in range(args.steps):
        dt, _ = cpu_baseline(w, threads)
        tot += dt
    pairs = w["pairs_factor"] + w["pairs_solve"]
    v = pairs * args.steps / tot
    line = {"impl": "reference", "metric": "(x)(+) pairs/s in mlu + lmul! (config 2)", "value": v,
            "unit": "pairs/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic (seeded, config 2 shapes)",
            "config": {"workload": w["name"], "semiring": "MinPlus", "n": w["n"], "nrhs": w["k"]},
            "cpu_baseline": {"value": v, "unit": "pairs/s", "cores": threads, "kind": "port",
                             "sample": "full config-2 workload per step (assembly + factorization + lmul!), "
                                       "oracle/ C restatement with OpenMP; Julia is not installed"},
            "e2e": {"value": v, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_once():
    """The workload's step twice (warm-up, then the step an ncu capture selects with -s / -c), nothing timed."""
    import torch

    import pathpack_b200 as pp

    w = config2(0)
    F = pp.B200SLU(pp.MinPlus(), np.float64, w["S"], device=0)
    nz_d = torch.from_numpy(w["nz"]).to("cuda:0")
    B0 = torch.from_numpy(np.ascontiguousarray(w["B"].T)).to("cuda:0")
    F.assemble_csc(w["cp"], w["rv"], w["nz"])
    for _ in range(2):
        F.update_values(nz_d)
        F.factor()
        Bw = B0.clone()
        pp.lmul_(F, Bw.T)
    torch.cuda.synchronize()
    F.close()


def run_ours(args, rank, world, local):
    import torch

    import pathpack_b200 as pp

    dist = world > 1
    if dist:
        import torch.distributed as tdist
    dev = local
    torch.cuda.set_device(dev)
    from pathpack_b200.panels import column_panels, join_group

    # one job on all ranks (strong scaling): the same matrix and right-hand sides everywhere; the factorization
    # is split (every rank factors its part of the bottom of the tree, NCCL broadcasts exchange the parts, every
    # rank factors the top) and each rank solves its own column panel of B
    w = config2(0)
    n, k = w["n"], w["k"]
    pc0, kw = column_panels(k, world)[rank]
    S = w["S"]
    F = pp.B200SLU(pp.MinPlus(), np.float64, S, device=dev)
    if dist:
        join_group(F)
    F.assemble_csc(w["cp"], w["rv"], w["nz"]).factor()
    stream = torch.cuda.ExternalStream(F.stream(), device=dev)
    nz_d = torch.from_numpy(w["nz"]).to(f"cuda:{dev}")
    B0 = torch.from_numpy(np.ascontiguousarray(w["B"][:, pc0:pc0 + kw].T)).to(f"cuda:{dev}")  # (kw, n): n x kw
    Bw = torch.empty_like(B0)
    # this rank's algorithmic pairs: the factorization once for the job (rank 0), lmul! of its columns
    nn_, na_ = S.nn.astype(np.float64), S.na.astype(np.float64)
    u_full = float((nn_ * (nn_ - 1) / 2 + nn_ * na_).sum())
    src = np.array([int(np.flatnonzero(w["B"][:, c] == 0.0)[0]) for c in range(pc0, pc0 + kw)], dtype=np.int64)
    pairs_rank = (w["pairs_factor"] if rank == 0 else 0.0) + S.rootpath_pairs(S.invp[src]) + kw * u_full

    def step_calls():
        # the step as separate C-ABI calls, everything enqueued on the library's stream (no host wait)
        F.update_values(nz_d)  # 5 fills + the assembly kernel
        F.factor(sync=False)
        with torch.cuda.stream(stream):
            Bw.copy_(B0)
        F._solve(Bw.T, True, sync=False)

    if dist:
        # joined handles run call by call (the factorization's broadcasts are not captured into a graph)
        plan = None
        F.factor()
        launches_per_step = 6 + F.stats()["kernel_launches"]
        F._solve(Bw.T, True)
        launches_per_step += F.stats()["kernel_launches"]

        def step():
            step_calls()
    else:
        # the timed step: the same calls captured once as a CUDA graph by the library (pp_plan_lmul: re-assembly
        # from the device weights, factorization, lmul! of B0 into Bw), so that one graph launch enqueues the
        # whole step and the host's speed does not enter the device time
        plan = F.plan_lmul(nz_d, B0.T, Bw.T)
        launches_per_step = plan.launches

        def step():
            plan.launch()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gidx = int(vis.split(",")[dev]) if vis else dev
    # the clock sampler starts before the warm-up, so that its start (NVML initialisation) is not inside the
    # timed region; every step is bracketed by its own pair of events on the library's stream and the host
    # time to enqueue it is recorded, so that a stall shows as one slow step or as host-bound enqueueing
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    enqueue_ms = []
    with Clocks(gidx) as clk:
        for _ in range(args.warmup):
            step()
        F.sync()
        torch.cuda.synchronize(dev)
        if dist:
            tdist.barrier()
        torch.cuda.synchronize(dev)
        evs[0].record(stream)
        for i in range(args.steps):
            t0 = time.perf_counter()
            step()
            evs[i + 1].record(stream)
            enqueue_ms.append(1e3 * (time.perf_counter() - t0))
        torch.cuda.synchronize(dev)
        F.sync()  # reports a device error of the timed steps
    step_ms = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
    e0, e1 = evs[0], evs[-1]
    launches = launches_per_step * args.steps
    # for comparison: the same steps enqueued call by call (not part of the value)
    for _ in range(2):
        step_calls()
    F.sync()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record(stream)
    for _ in range(args.steps):
        step_calls()
    c1.record(stream)
    F.sync()
    calls_ms = c0.elapsed_time(c1) / args.steps
    ms = e0.elapsed_time(e1)
    clocks = clk.summary()
    if dist:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        ms = float(t.item())
    pairs = _sum_over_ranks(pairs_rank, dev, world)  # = pairs_factor + pairs_solve of the one job
    value = pairs * args.steps / (ms / 1e3)

    # e2e: host CSC + pinned host B through the C ABI, H2D and D2H inside each timed step
    Bh = torch.empty((kw, n), dtype=torch.float64, pin_memory=True)
    Bh_np = Bh.numpy()
    Bsrc = np.ascontiguousarray(w["B"][:, pc0:pc0 + kw].T)
    e2e_t = 0.0
    e2e_steps = []
    for it in range(args.warmup + args.steps):
        np.copyto(Bh_np, Bsrc)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        F.update_values(w["nz"]).factor(sync=False)  # host weights: H2D inside, re-assembled on the device
        pp.lmul_(F, Bh_np.T)  # host B: H2D and D2H inside; returns when the result is in host memory
        t1 = time.perf_counter()
        if it >= args.warmup:
            e2e_t += t1 - t0
            e2e_steps.append(1e3 * (t1 - t0))
    if dist:
        t = torch.tensor([e2e_t], device=f"cuda:{dev}")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        e2e_t = float(t.item())
    h2d = w["nz"].nbytes + n * kw * 8  # per rank
    d2h = n * kw * 8

    # roofline of the dominant kernel class, measured with CUDA events on the library's stream over K steps
    F.set_profile(True)
    for _ in range(args.steps):
        step_calls()  # the profiler brackets the library's launches with events: call by call, not the graph
    F.sync()
    prof = F.profile()
    F.set_profile(False)
    pk, src = peaks()
    top = max(prof.items(), key=lambda kv: kv[1]["ms"])
    name, d = top
    per_launch_s = d["ms"] / 1e3 / d["launches"]
    # the dominant kernel (the top factorization) is bound by its ALU issue rate along the tree's critical
    # path, not by HBM: its fraction is (x)(+) pairs per second against the nominal Float64 ALU pair peak
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    apeak = alu_peak("MinPlus", np.float64, sms, float(pk.get("sm_max_mhz", 1965.0)))
    achieved = d["pairs"] / d["launches"] / per_launch_s
    gbs = d["bytes"] / d["launches"] / per_launch_s / 1e9
    roof = {"kernel": name, "bound": "alu", "achieved": achieved, "peak": apeak, "unit": "pairs/s",
            "frac": achieved / apeak,
            "peak_source": "nominal Float64 ALU issue rate: SMs x max SM clock (MEASURED_PEAKS sm_max_mhz) x 64 "
                           "lanes / 2 instructions per (x)(+) pair",
            "traffic": ncu_traffic(args.traffic_csv, name),
            "traffic_source": args.traffic_csv or "none given (--traffic-csv); see profiles/ for the ncu capture",
            "hbm_achieved_GB_per_s": gbs, "hbm_peak_GB_per_s": float(pk["hbm_gbs"]),
            "hbm_frac": gbs / float(pk["hbm_gbs"]), "hbm_peak_source": src,
            "algorithmic_bytes_per_launch": d["bytes"] / d["launches"],
            "pairs_per_launch": d["pairs"] / d["launches"],
            "launches_per_step": d["launches"] / args.steps, "ms_per_step": d["ms"] / args.steps}
    kernels = {k_: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps,
                    "GB_per_s": v["bytes"] / (v["ms"] / 1e3) / 1e9 if v["ms"] > 0 else 0.0,
                    "Tpairs_per_s": v["pairs"] / (v["ms"] / 1e3) / 1e12 if v["ms"] > 0 else 0.0}
               for k_, v in prof.items()}

    # mstar of config 4 on the same N GPUs, its columns split into one contiguous panel per rank (strong scaling;
    # every rank factors the same matrix): the metric's "mstar wall-s at 1/2/4/8 B200"
    mstar = None
    if not args.no_mstar:
        ms4 = measure_star("config4", rank, world, dev, max(3, args.steps // 2), args.warmup, e2e=False)
        mstar = {"workload": STAR["config4"]["name"], "wall_s": ms4["wall_s"], "value": ms4["value"],
                 "unit": "pairs/s", "n_gpus": world, "scaling": "strong",
                 "parallelism": ms4["parallelism"], "columns_per_rank": ms4["columns_per_rank"],
                 "pairs_per_step": ms4["pairs_per_step"], "output": "device-resident",
                 "symbolic_s_host": ms4["symbolic_s"], "clocks": ms4["clocks"]}

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            threads = os.cpu_count() or 1
            dt, Xc = cpu_baseline(w, threads)
            # the device result of the last step against the oracle (bit-exact for MinPlus)
            got = Bw.T.cpu().numpy()  # the whole of B at N = 1
            cpu = {"value": pairs / dt, "unit": "pairs/s", "cores": threads, "kind": "port",
                   "sample": "one full config-2 step (assembly + factorization + lmul!) with the oracle/ C "
                             "restatement on %d threads; Julia is not installed" % threads,
                   "seconds": dt, "matches_device_bitwise": bool(np.array_equal(got, Xc))}
        line = {"metric": "(x)(+) pairs/s in mlu + lmul! (config 2)", "value": value, "unit": "pairs/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic (seeded; config 2 shapes: 256x256 grid digraph, U[1,10) weights, unit columns)",
                "config": {"workload": w["name"], "semiring": "MinPlus", "n": n, "nrhs": k, "nf": w["S"].nf,
                           "pairs_per_step": pairs, "pairs_factor": w["pairs_factor"],
                           "pairs_solve": w["pairs_solve"], "columns_per_rank": [c for _, c in column_panels(k, world)],
                           "parallelism": ("one GPU" if world == 1 else
                                           "one job: the bottom of the tree split over the GPUs (its parts "
                                           "exchanged by NCCL broadcasts), the top factored on every GPU, B split "
                                           "into column panels"),
                           "l2": "inputs larger than L2 (B 134 MB + factor + workspace)"},
                "e2e": {"value": pairs * args.steps / e2e_t, "unit": "pairs/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": 1e3 * e2e_t / args.steps,
                        "step_ms_min": min(e2e_steps), "step_ms_median": float(np.median(e2e_steps)),
                        "clock": "host wall clock per step (perf_counter), summed over the K steps"},
                "step_ms": {"median": float(np.median(step_ms)), "min": min(step_ms), "max": max(step_ms),
                            "clock": "CUDA events on the library's stream around each timed step",
                            "step": ("one launch of the library's captured plan (pp_plan_lmul): re-assembly, "
                                     "factorization, lmul!" if world == 1 else
                                     "the C-ABI calls: re-assembly, split factorization, lmul! of the rank's panel"),
                            "call_by_call_ms_per_step": calls_ms},
                "enqueue_ms": {"median": float(np.median(enqueue_ms)), "max": max(enqueue_ms),
                               "clock": "host perf_counter around enqueueing each timed step"},
                "gpu_launches": launches, "roofline": roof, "kernels": kernels, "clocks": clocks,
                "cpu_baseline": cpu, "mstar": mstar}
        print(json.dumps(line), flush=True)
    if plan is not None:
        plan.close()
    F.close()


def _max_over_ranks(x, dev, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as tdist

    t = torch.tensor([float(x)], device=f"cuda:{dev}")
    tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(x, dev, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as tdist

    t = torch.tensor([float(x)], device=f"cuda:{dev}", dtype=torch.float64)
    tdist.all_reduce(t, op=tdist.ReduceOp.SUM)
    return float(t.item())


def _gpu_index(dev):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return int(vis.split(",")[dev]) if vis else dev


def _roofline_alu(prof, steps, semiring, dtype, pk):
    """The kernel class with the largest share of device time: its (x)(+) pairs per second against the
    nominal ALU issue peak at the measured maximum SM clock (these kernels are ALU- or latency-bound)."""
    import torch

    name, d = max(prof.items(), key=lambda kv: kv[1]["ms"])
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    peak = alu_peak(semiring, dtype, sms, float(pk.get("sm_max_mhz", 1965.0)))
    achieved = d["pairs"] / (d["ms"] / 1e3) if d["ms"] > 0 else 0.0
    return {"kernel": name, "bound": "alu", "achieved": achieved, "peak": peak, "unit": "pairs/s",
            "frac": achieved / peak, "traffic": None, "peak_source": "nominal ALU issue rate "
            "(SMs x max SM clock x lanes / instructions per pair)", "ms_per_step": d["ms"] / steps,
            "launches_per_step": d["launches"] / steps,
            "GB_per_s": d["bytes"] / (d["ms"] / 1e3) / 1e9 if d["ms"] > 0 else 0.0}


def measure_star(key, rank, world, dev, steps, warmup, e2e=True, cpu=False, w=None, columns=None):
    """mlu + this rank's column panel of Matrix(F) for a star workload; returns the numbers of one rank (times
    already the max over ranks)."""
    import torch

    import pathpack_b200 as pp
    from pathpack_b200._lib import PP_DEVICE, PP_HOST, check
    from pathpack_b200.panels import column_panels

    w = w or star_workload(key)
    n, S = w["n"], w["S"]
    sr = getattr(pp, w["semiring"])()
    tdt = {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64}[np.dtype(w["dtype"])]
    es = np.dtype(w["dtype"]).itemsize
    col0, ncols = column_panels(n, world)[rank]
    if columns:  # a smaller case of the same kernels (profiling captures): the first columns of the panel
        ncols = min(ncols, int(columns))
    F = pp.B200SLU(sr, w["dtype"], S, device=dev)
    if world > 1:  # the factorization split over the ranks (NCCL), every rank ends with the whole factor
        from pathpack_b200.panels import join_group

        join_group(F)
    F.assemble_csc(w["cp"], w["rv"], w["nz"]).factor()
    stream = torch.cuda.ExternalStream(F.stream(), device=dev)
    nz_d = torch.from_numpy(w["nz"]).to(f"cuda:{dev}")
    out = torch.empty((max(ncols, 1), n), dtype=tdt, device=f"cuda:{dev}").t()  # column-major n x ncols
    lib = pp.lib()

    def step():
        F.update_values(nz_d)
        F.factor(sync=False)
        check(lib.pp_star(F._h, out.data_ptr(), n, col0, ncols, PP_DEVICE), F._h)

    F.update_values(nz_d)
    F.factor()
    launches = 6 + F.stats()["kernel_launches"]
    check(lib.pp_star(F._h, out.data_ptr(), n, col0, ncols, PP_DEVICE), F._h)
    F.sync()
    launches += F.stats()["kernel_launches"]
    for _ in range(warmup):
        step()
    F.sync()
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as tdist

        tdist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(_gpu_index(dev)) as clk:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        F.sync()
    ms = _max_over_ranks(e0.elapsed_time(e1), dev, world)
    pairs_rank = (w["pairs_factor"] if rank == 0 else 0.0) + star_pairs(w, col0, ncols)
    pairs = _sum_over_ranks(pairs_rank, dev, world)  # the job's factorization once, every rank's columns
    r = {"ms_per_step": ms / steps, "wall_s": ms / steps / 1e3, "pairs_per_step": pairs,
         "value": pairs * steps / (ms / 1e3), "launches": launches * steps, "clocks": clk.summary(),
         "columns_per_rank": [min(c, int(columns)) if columns else c for _, c in column_panels(n, world)],
         "symbolic_s": w["symbolic_s"],
         "parallelism": ("one GPU" if world == 1 else "the bottom of the tree split over the GPUs (NCCL broadcasts), "
                         "the top factored on every GPU, column panels of A*")}
    if e2e:
        # host weights in, the rank's panel of the star out into pinned host memory, both inside the call
        host = torch.empty((max(ncols, 1), n), dtype=tdt, pin_memory=True)
        hv = host.numpy()
        tot = []
        for it in range(1 + min(steps, 3)):
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            F.update_values(w["nz"]).factor(sync=False)
            check(lib.pp_star(F._h, hv.ctypes.data, n, col0, ncols, PP_HOST), F._h)
            if it:
                tot.append(time.perf_counter() - t0)
        t = _max_over_ranks(sum(tot), dev, world)
        r["e2e"] = {"value": pairs * len(tot) / t, "unit": "pairs/s", "wall_s": t / len(tot),
                    "h2d_bytes_per_step": int(w["nz"].nbytes), "d2h_bytes_per_step": int(n * ncols * es),
                    "steps": len(tot), "clock": "host wall clock per call (perf_counter), max over ranks"}
        del host, hv
    F.set_profile(True)
    step()
    F.sync()
    r["prof"] = F.profile()
    F.set_profile(False)
    if cpu and rank == 0 and world == 1:
        r["cpu_baseline"] = star_cpu(w, torch_out=out)
    F.close()
    del out
    torch.cuda.empty_cache()
    return r


def star_cpu(w, torch_out=None, threads=None):
    """The oracle on a bounded sample: mlu, then columns 0 .. m-1 of A* as lmul!(F, I[:, 0:m]); pairs/s."""
    import pathpack_b200 as pp
    from oracle.oracle import OracleLU

    threads = threads or os.cpu_count() or 1
    sr = getattr(pp, w["semiring"])()
    n, m = w["n"], min(w["cpu_cols"], w["n"])
    B = np.full((n, m), sr.zero(w["dtype"]), dtype=w["dtype"], order="F")
    B[np.arange(m), np.arange(m)] = sr.one(w["dtype"])
    t0 = time.perf_counter()
    O = OracleLU(w["semiring"], w["dtype"], w["S"]).assemble(w["cp"], w["rv"], w["nz"]).factor(threads)
    X = O.lmul(B, threads)
    dt = time.perf_counter() - t0
    pairs = w["pairs_factor"] + star_pairs(w, 0, m)
    r = {"value": pairs / dt, "unit": "pairs/s", "cores": threads, "kind": "port", "seconds": dt,
         "sample": "mlu plus columns 0..%d of A* (lmul! of the unit columns) with the oracle/ C restatement on %d "
                   "threads; Julia is not installed" % (m - 1, threads)}
    if torch_out is not None:
        r["matches_device_bitwise"] = bool(np.array_equal(torch_out[:, :m].cpu().numpy(), X))
    return r


def run_star(args, rank, world, local):
    import torch

    torch.cuda.set_device(local)
    key = args.workload
    w = star_workload(key)
    r = measure_star(key, rank, world, local, args.steps, args.warmup, e2e=not args.no_e2e,
                     cpu=not args.no_cpu_baseline and not args.columns, w=w, columns=args.columns)
    if rank != 0:
        return
    pk, _ = peaks()
    roof = _roofline_alu(r["prof"], 1, w["semiring"], w["dtype"], pk)
    kernels = {k_: {"ms_per_step": v["ms"], "launches_per_step": v["launches"],
                    "Tpairs_per_s": v["pairs"] / (v["ms"] / 1e3) / 1e12 if v["ms"] > 0 else 0.0}
               for k_, v in r["prof"].items()}
    line = {"metric": "(x)(+) pairs/s in mlu + Matrix(F) (%s); mstar wall-s" % key, "value": r["value"],
            "unit": "pairs/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"], "mstar_wall_s": r["wall_s"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f64" if np.dtype(w["dtype"]) == np.float64 else "f32",
            "data": "synthetic (seeded, %s shapes)" % key,
            "config": {"workload": w["name"], "semiring": w["semiring"], "n": w["n"], "nf": w["S"].nf,
                       "pairs_per_step": r["pairs_per_step"], "columns_per_rank": r["columns_per_rank"],
                       "parallelism": "column panels of A* (factor replicated on every GPU)",
                       "output": "device-resident column panels",
                       "symbolic_s_host": r["symbolic_s"],
                       "l2": "output panels larger than L2"},
            "gpu_launches": r["launches"], "roofline": roof, "kernels": kernels, "clocks": r["clocks"]}
    if "e2e" in r:
        line["e2e"] = r["e2e"]
    if "cpu_baseline" in r:
        line["cpu_baseline"] = r["cpu_baseline"]
    print(json.dumps(line), flush=True)


# config 5: the dense kernels alone
KERNELS = {
    "config5a": dict(semiring="MinPlus", dtype=np.int32, name="batched getrf, 4096 x 128x128 MinPlus Int32"),
    "config5b-i32": dict(semiring="MinPlus", dtype=np.int32, name="semiring GEMM 8192^3 MinPlus Int32"),
    "config5b-f32": dict(semiring="MinPlus", dtype=np.float32, name="semiring GEMM 8192^3 MinPlus Float32"),
    "config5b-f64": dict(semiring="PlusProd", dtype=np.float64, name="semiring GEMM 8192^3 PlusProd Float64"),
}


def kernel_inputs(key, rng):
    """Host inputs of a config-5 workload, seeded, as BASELINE.json specifies them (column-major)."""
    w = KERNELS[key]
    if key == "config5a":
        count, n = 4096, 128
        A = rng.integers(1, 1001, size=(count, n, n)).astype(np.int32)
        A[rng.random(A.shape) < 0.4] = np.iinfo(np.int32).max
        A[:, np.arange(n), np.arange(n)] = 0
        return dict(A=A, n=n, count=count, pairs=count * sum(q * q for q in range(n)))
    N = 8192
    if w["dtype"] == np.int32:
        A = rng.integers(1, 1001, size=(N, N)).astype(np.int32)
        B = rng.integers(1, 1001, size=(N, N)).astype(np.int32)
        C = np.full((N, N), np.iinfo(np.int32).max, np.int32)
    elif w["dtype"] == np.float32:
        A = rng.random((N, N), dtype=np.float32)
        B = rng.random((N, N), dtype=np.float32)
        C = np.full((N, N), np.inf, np.float32)
    else:
        A = rng.random((N, N)) / N
        B = rng.random((N, N)) / N
        C = np.zeros((N, N))
    return dict(A=A, B=B, C=C, N=N, pairs=float(N) ** 3)


def run_kernel(args, rank, world, local):
    """Config 5: one launch of pp_getrf_batched or pp_gemm per step on device-resident inputs; with N ranks each
    GPU runs its own instance (weak scaling, no collective)."""
    import torch

    import pathpack_b200 as pp
    from pathpack_b200._lib import check
    from pathpack_b200.semiring import DTYPES

    torch.cuda.set_device(local)
    key = args.workload
    w = KERNELS[key]
    sr = getattr(pp, w["semiring"])()
    dt = DTYPES[np.dtype(w["dtype"])]
    rng = np.random.default_rng(15 + rank)
    x = kernel_inputs(key, rng)
    dev = f"cuda:{local}"
    lib = pp.lib()
    st = torch.cuda.Stream(device=local)
    if key == "config5a":
        A0 = torch.from_numpy(x["A"]).to(dev)
        Aw = torch.empty_like(A0)
        nbytes = 2 * A0.numel() * 4

        def launch():
            check(lib.pp_getrf_batched(sr.id, dt, x["n"], x["count"], Aw.data_ptr(), st.cuda_stream))

        def reset():
            with torch.cuda.stream(st):
                Aw.copy_(A0)
    else:
        N = x["N"]
        # a column-major N x N matrix M is the row-major tensor M.T
        A = torch.from_numpy(np.ascontiguousarray(x["A"].T)).to(dev)
        B = torch.from_numpy(np.ascontiguousarray(x["B"].T)).to(dev)
        C0 = torch.from_numpy(np.ascontiguousarray(x["C"].T)).to(dev)
        Cw = torch.empty_like(C0)
        es = A.element_size()
        nbytes = es * 4 * N * N  # A and B read, C read and written

        def launch():
            check(lib.pp_gemm(sr.id, dt, N, N, N, Cw.data_ptr(), N, A.data_ptr(), N, B.data_ptr(), N, st.cuda_stream))

        def reset():
            with torch.cuda.stream(st):
                Cw.copy_(C0)
    # each step: the input is reset (outside the events), then the kernel is timed alone on its stream
    for _ in range(args.warmup):
        reset()
        launch()
    torch.cuda.synchronize(local)
    if world > 1:
        import torch.distributed as tdist

        tdist.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with Clocks(_gpu_index(local)) as clk:
        for e0, e1 in evs:
            reset()
            e0.record(st)
            launch()
            e1.record(st)
        torch.cuda.synchronize(local)
    ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in evs), local, world)
    value = x["pairs"] * world * args.steps / (ms / 1e3)
    # e2e: pinned host inputs uploaded, the kernel, the result downloaded, all inside each timed call
    if key == "config5a":
        hin = torch.from_numpy(x["A"]).pin_memory()
        hout = torch.empty_like(hin).pin_memory()
        h2d, d2h = hin.numel() * 4, hin.numel() * 4

        def e2e_call():
            with torch.cuda.stream(st):
                Aw.copy_(hin, non_blocking=True)
            launch()
            with torch.cuda.stream(st):
                hout.copy_(Aw, non_blocking=True)
            st.synchronize()
    else:
        hA = torch.from_numpy(np.ascontiguousarray(x["A"].T)).pin_memory()
        hB = torch.from_numpy(np.ascontiguousarray(x["B"].T)).pin_memory()
        hC = torch.from_numpy(np.ascontiguousarray(x["C"].T)).pin_memory()
        hout = torch.empty_like(hC).pin_memory()
        h2d, d2h = 3 * hA.numel() * hA.element_size(), hA.numel() * hA.element_size()

        def e2e_call():
            with torch.cuda.stream(st):
                A.copy_(hA, non_blocking=True)
                B.copy_(hB, non_blocking=True)
                Cw.copy_(hC, non_blocking=True)
            launch()
            with torch.cuda.stream(st):
                hout.copy_(Cw, non_blocking=True)
            st.synchronize()
    e2e_call()
    tot = 0.0
    ne = min(args.steps, 3)
    for _ in range(ne):
        torch.cuda.synchronize(local)
        t0 = time.perf_counter()
        e2e_call()
        tot += time.perf_counter() - t0
    tot = _max_over_ranks(tot, local, world)
    if rank != 0:
        return
    pk, _ = peaks()
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    peak = alu_peak(w["semiring"], w["dtype"], sms, float(pk.get("sm_max_mhz", 1965.0)))
    per_launch = ms / 1e3 / args.steps
    dmma = key == "config5b-f64"
    roof = {"kernel": "getrf_reg_kernel" if key == "config5a" else ("gemm_dmma_tma_kernel" if dmma else "gemm_kernel"),
            "bound": "tensor" if dmma else "alu",
            "achieved": x["pairs"] / per_launch, "peak": peak, "unit": "pairs/s", "frac": x["pairs"] / per_launch / peak,
            "traffic": None,
            "peak_source": ("nominal FP64 tensor (DMMA) rate: SMs x max SM clock x 64 multiply-adds per clock" if dmma
                            else "nominal ALU issue rate (SMs x max SM clock x lanes / instructions per pair)"),
            "hbm_GB_per_s": nbytes / per_launch / 1e9, "hbm_frac": nbytes / per_launch / 1e9 / float(pk["hbm_gbs"])}
    line = {"metric": "(x)(+) pairs/s (%s)" % key, "value": value, "unit": "pairs/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": {np.dtype(np.int32): "int32", np.dtype(np.float32): "f32",
                                                               np.dtype(np.float64): "f64"}[np.dtype(w["dtype"])],
            "data": "synthetic (seeded, BASELINE config 5 distributions)",
            "config": {"workload": w["name"], "semiring": w["semiring"], "pairs_per_step": x["pairs"],
                       "parallelism": "independent instance per GPU",
                       "l2": "inputs larger than L2; the input is reset by a device copy before each timed launch"},
            "e2e": {"value": x["pairs"] * world * ne / tot, "unit": "pairs/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h), "ms_per_step": 1e3 * tot / ne,
                    "clock": "host wall clock per call (perf_counter), pinned host buffers"},
            "gpu_launches": args.steps, "roofline": roof, "clocks": clk.summary()}
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = kernel_cpu(key, x)
    print(json.dumps(line), flush=True)


def kernel_cpu(key, x, threads=None):
    """The oracle's getrf / GEMM on a bounded sample of the same inputs: pairs/s."""
    from oracle import oracle as orc

    threads = threads or os.cpu_count() or 1
    w = KERNELS[key]
    if key == "config5a":
        m = x["count"]  # the whole batch: a fraction of a second on the host cores
        A = np.ascontiguousarray(x["A"][:m])
        t0 = time.perf_counter()
        orc.getrf_batched(w["semiring"], A, threads)
        dt = time.perf_counter() - t0
        pairs, sample = m * sum(q * q for q in range(x["n"])), "%d of the 4096 blocks" % m
    else:
        cols = 512
        C = np.asfortranarray(x["C"][:, :cols])
        A, B = np.asfortranarray(x["A"]), np.asfortranarray(x["B"][:, :cols])
        t0 = time.perf_counter()
        orc.gemm(w["semiring"], C, A, B, threads)
        dt = time.perf_counter() - t0
        pairs, sample = float(x["N"]) * x["N"] * cols, "C[:, 0:%d] (8192 x %d x 8192)" % (cols, cols)
    return {"value": pairs / dt, "unit": "pairs/s", "cores": threads, "kind": "port", "seconds": dt,
            "sample": sample + " with the oracle/ C restatement on %d threads; Julia is not installed" % threads}


def run_reference_workload(args, rank, world):
    """--impl reference for the star and kernel workloads: the oracle on the host cores, rank 0 only."""
    if rank != 0:
        return
    tot, cpu = 0.0, None
    if args.workload in STAR:
        w = star_workload(args.workload)
        for _ in range(args.warmup):
            star_cpu(w)
        vals = [star_cpu(w) for _ in range(args.steps)]
        unit_dtype = w["dtype"]
    else:
        w = KERNELS[args.workload]
        x = kernel_inputs(args.workload, np.random.default_rng(15))
        for _ in range(args.warmup):
            kernel_cpu(args.workload, x)
        vals = [kernel_cpu(args.workload, x) for _ in range(args.steps)]
        unit_dtype = w["dtype"]
    v = float(np.median([c["value"] for c in vals]))
    tot = sum(c["seconds"] for c in vals)
    cpu = dict(vals[-1])
    cpu["value"] = v
    line = {"impl": "reference", "metric": ("(x)(+) pairs/s in mlu + Matrix(F) (%s); mstar wall-s" % args.workload
                                            if args.workload in STAR else "(x)(+) pairs/s (%s)" % args.workload),
            "value": v, "unit": "pairs/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.workload in STAR else "weak", "vs_baseline": None,
            "dtype": str(np.dtype(unit_dtype)), "data": "synthetic (seeded, %s shapes)" % args.workload,
            "config": {"workload": w["name"], "semiring": w["semiring"]}, "cpu_baseline": cpu,
            "e2e": {"value": v, "unit": "pairs/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--once", action="store_true",
                    help="one warm-up step and one step of the workload, no timing line (for ncu captures)")
    ap.add_argument("--workload", default="config2", choices=["config2"] + list(STAR) + list(KERNELS),
                    help="config2 (default, the headline line), a star workload (config1/3/4, column panels "
                         "over the ranks) or a config-5 kernel")
    ap.add_argument("--no-e2e", action="store_true", help="star workloads: skip the host-output e2e calls")
    ap.add_argument("--no-mstar", action="store_true", help="config2: skip the config-4 mstar sub-measurement")
    ap.add_argument("--traffic-csv", default=None,
                    help="an ncu raw CSV export (ncu -i <rep> --page raw --csv) of this build: fills roofline.traffic")
    ap.add_argument("--columns", type=int, default=None,
                    help="star workloads: compute only the first C columns of each rank's panel (a smaller case "
                         "of the same kernels, for profiling captures; the line then covers those columns)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        if args.workload == "config2":
            run_reference(args, rank, world)
        else:
            run_reference_workload(args, rank, world)
        return
    if args.once:
        run_once()
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local)
        # NVLink SHARP off for the process group and the library's group (its kernels use no multicast either)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        if args.workload in STAR:
            run_star(args, rank, world, local)
        elif args.workload in KERNELS:
            run_kernel(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as tdist

            tdist.barrier()
            tdist.destroy_process_group()


if __name__ == "__main__":
    main()
