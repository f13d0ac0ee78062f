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

Multi-GPU (--gpus N under torchrun): each rank factors and solves its own independent instance (weak scaling,
no collective on the data path); value = all ranks' pairs / the slowest rank's time.

--impl reference runs the reference's CPU algorithm (the oracle: the C restatement of PATHPACK.jl's CPU path,
oracle/; Julia is not available here) on the host cores, on the same workload; rank 0 only.
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


def profiled_traffic(kernel):
    """DRAM bytes per launch of the kernel (dram__bytes_read.sum + dram__bytes_write.sum) from the committed ncu
    summary profiles/<kernel>_config2.md, or None."""
    path = os.path.join(REPO, "profiles", "%s_config2.md" % kernel.split("(")[0])
    if not os.path.exists(path):
        return None
    for line in open(path):
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":")[1])
    return None


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
            "ms_per_step": 1e3 * tot / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
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
    w = config2(rank)
    n, k = w["n"], w["k"]
    F = pp.B200SLU(pp.MinPlus(), np.float64, w["S"], device=dev)
    F.assemble_csc(w["cp"], w["rv"], w["nz"]).factor()
    stream = torch.cuda.ExternalStream(F.stream(), device=dev)
    nz_d = torch.from_numpy(w["nz"]).to(f"cuda:{dev}")
    B0 = torch.from_numpy(np.ascontiguousarray(w["B"].T)).to(f"cuda:{dev}")  # (k, n): column-major n x k
    Bw = torch.empty_like(B0)

    def step():
        # everything is enqueued on the library's stream: no host synchronisation inside the step
        F.update_values(nz_d)  # 5 fills + the assembly kernel
        F.factor(sync=False)
        with torch.cuda.stream(stream):
            Bw.copy_(B0)
        F._solve(Bw.T, True, sync=False)

    # the library's kernel launches of one step (the same every step): factorization + solve + 6 for the
    # re-assembly (stats() waits, so it is read outside the timed region)
    F.update_values(nz_d)
    F.factor()
    launches_per_step = 6 + F.stats()["kernel_launches"]
    with torch.cuda.stream(stream):
        Bw.copy_(B0)
    pp.lmul_(F, Bw.T)
    launches_per_step += F.stats()["kernel_launches"]
    for _ in range(args.warmup):
        step()
    F.sync()
    torch.cuda.synchronize(dev)
    if dist:
        tdist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    gidx = int(vis.split(",")[dev]) if vis else dev
    with Clocks(gidx) as clk:
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        F.sync()  # reports a device error of the timed steps
    launches = launches_per_step * args.steps
    ms = e0.elapsed_time(e1)
    clocks = clk.summary()
    if dist:
        t = torch.tensor([ms], device=f"cuda:{dev}")
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        ms = float(t.item())
    pairs = w["pairs_factor"] + w["pairs_solve"]
    value = pairs * world * args.steps / (ms / 1e3)

    # e2e: host CSC + pinned host B through the C ABI, H2D and D2H inside each timed step
    Bh = torch.empty((k, n), dtype=torch.float64, pin_memory=True)
    Bh_np = Bh.numpy()
    Bsrc = np.ascontiguousarray(w["B"].T)
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
    h2d = w["nz"].nbytes + n * k * 8
    d2h = n * k * 8

    # roofline of the dominant kernel class, measured with CUDA events on the library's stream over K steps
    F.set_profile(True)
    for _ in range(args.steps):
        step()
    F.sync()
    prof = F.profile()
    F.set_profile(False)
    pk, src = peaks()
    top = max(prof.items(), key=lambda kv: kv[1]["ms"])
    name, d = top
    per_launch_s = d["ms"] / 1e3 / d["launches"]
    achieved = d["bytes"] / d["launches"] / per_launch_s / 1e9
    roof = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": float(pk["hbm_gbs"]), "unit": "GB/s",
            "frac": achieved / float(pk["hbm_gbs"]), "traffic": profiled_traffic(name), "peak_source": src,
            "launches_per_step": d["launches"] / args.steps, "ms_per_step": d["ms"] / args.steps,
            "pairs_per_s": d["pairs"] / (d["ms"] / 1e3) if d["ms"] > 0 else 0.0}
    kernels = {k_: {"ms_per_step": v["ms"] / args.steps, "launches_per_step": v["launches"] / args.steps,
                    "GB_per_s": v["bytes"] / (v["ms"] / 1e3) / 1e9 if v["ms"] > 0 else 0.0,
                    "Tpairs_per_s": v["pairs"] / (v["ms"] / 1e3) / 1e12 if v["ms"] > 0 else 0.0}
               for k_, v in prof.items()}

    line = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            threads = os.cpu_count() or 1
            dt, Xc = cpu_baseline(w, threads)
            # the device result of the last step against the oracle (bit-exact for MinPlus)
            got = Bw.T.cpu().numpy()
            cpu = {"value": pairs / dt, "unit": "pairs/s", "cores": threads, "kind": "port",
                   "sample": "one full config-2 step (assembly + factorization + lmul!) with the oracle/ C "
                             "restatement on %d threads; Julia is not installed" % threads,
                   "seconds": dt, "matches_device_bitwise": bool(np.array_equal(got, Xc))}
        line = {"metric": "(x)(+) pairs/s in mlu + lmul! (config 2)", "value": value, "unit": "pairs/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
                "data": "synthetic (seeded; config 2 shapes: 256x256 grid digraph, U[1,10) weights, unit columns)",
                "config": {"workload": w["name"], "semiring": "MinPlus", "n": n, "nrhs": k, "nf": w["S"].nf,
                           "pairs_per_step_per_gpu": pairs, "pairs_factor": w["pairs_factor"],
                           "pairs_solve": w["pairs_solve"], "parallelism": "independent instance per GPU",
                           "l2": "inputs larger than L2 (B 134 MB + factor + workspace)"},
                "e2e": {"value": pairs * world * args.steps / e2e_t, "unit": "pairs/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": d2h, "ms_per_step": 1e3 * e2e_t / args.steps,
                        "step_ms_min": min(e2e_steps), "step_ms_median": float(np.median(e2e_steps)),
                        "clock": "host wall clock per step (perf_counter), summed over the K steps"},
                "gpu_launches": launches, "roofline": roof, "kernels": kernels, "clocks": clocks,
                "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    F.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--once", action="store_true",
                    help="one warm-up step and one step of the workload, no timing line (for ncu captures)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.once:
        run_once()
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as tdist

            tdist.barrier()
            tdist.destroy_process_group()


if __name__ == "__main__":
    main()
