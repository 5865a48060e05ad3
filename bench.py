#!/usr/bin/env python
"""Benchmark of the distributed CSR x dense SpMM (the hot path of DistSpMM) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload: R-MAT scale 20, edge factor 16,
(a,b,c,d) = (.57,.19,.19,.05), symmetrised, deduplicated, no self-loops (31.4 M nnz),
values U(0,1); dense B 1,048,576 x 128 fp32 U(-1,1); 1-D row partition over the ranks,
T = 4 tiles per rank, HSDMA allocation (task_dist 2), adaptive fetch (comm_type 2).
All inputs are seeded synthetic data generated here. The matrix is fixed as N grows
(strong scaling, as the reference partitions one matrix).

A step is one distributed SpMM C = A.B over the whole matrix: every rank fetches its
needed remote B rows (copy-engine bulk copies / NVLink gather kernels) and runs its
SpMM segments. Metric: GFLOPS = 2.nnz.dims / t, t = device time of a step (CUDA events
on the launching stream, mean over K steps, max over ranks). L2 is flushed between steps
(a 512 MiB write outside the timed events). `e2e` times the same steps through the C ABI
from pinned host memory: H2D of the rank's owned B tiles, the step, D2H of its C rows, run
back to back with the upload of step i+1 overlapping the download of step i.

`--impl reference` times the CPU CSR x dense loop of the oracle (the reference has no CPU
implementation of the path: its SpMM is cuSPARSE) with all host threads, on rank 0.
"""
from __future__ import annotations

import argparse
import contextlib
import csv
import datetime
import io
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "SpMM GFLOPS (2*nnz*N/t)"
UNIT = "GFLOPS"


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--matrix", choices=["rmat", "stencil27", "uniform"], default="rmat",
                    help="rmat: configurations 1/2/5; stencil27: configuration 3; uniform: configuration 4")
    ap.add_argument("--scale", type=int, default=20, help="R-MAT scale")
    ap.add_argument("--grid", type=int, default=160, help="stencil grid edge (160 -> 4,096,000 rows)")
    ap.add_argument("--rows", type=int, default=1 << 22, help="uniform matrix rows")
    ap.add_argument("--nnz-per-row", type=int, default=32, help="uniform matrix nonzeros per row")
    ap.add_argument("--dims", type=int, default=128)
    ap.add_argument("--n-rolls", type=int, default=4)
    ap.add_argument("--task-dist", type=int, default=2)
    ap.add_argument("--comm-type", type=int, default=2)
    ap.add_argument("--partition", choices=["rows", "balanced"], default="balanced",
                    help="A rows per rank: the reference's equal-row split or work-balanced (nnz + rows)")
    ap.add_argument("--fetch-scope", choices=["node", "rank"], default="rank",
                    help="remote B rows fetched: the node union of all ranks' needs (reference) or this rank's own")
    ap.add_argument("--pipeline", choices=["auto", "rows", "split"], default="auto",
                    help="phases: whole rows after their last fetch, nonzeros per ring position, or per matrix")
    ap.add_argument("--fetch-streams", type=int, default=4, help="concurrent fetch streams (nvlink_num_producers)")
    ap.add_argument("--platform", choices=["h100", "a800", "b200"], default="b200",
                    help="adaptive selector constants (comm_type 2); b200 = the NVLink 5 fit of comm_test")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-flush", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="short run for a profiler: warmup + steps only, no e2e / CPU baseline / clocks")
    return ap.parse_args(argv)


@contextlib.contextmanager
def stdout_to_stderr():
    """Point file descriptor 1 at stderr for the duration (output of native libraries too)."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def workload_name(a):
    if a.matrix == "stencil27":
        return f"stencil{a.grid}_n{a.dims}"
    if a.matrix == "uniform":
        return f"uniform{a.rows}x{a.nnz_per_row}_n{a.dims}"
    return f"rmat{a.scale}_n{a.dims}"


def matrix_desc(a):
    if a.matrix == "stencil27":
        return f"27-point stencil on a {a.grid}^3 grid, lexicographic; diagonal 26, off-diagonals U(-1,0)"
    if a.matrix == "uniform":
        return f"uniform random {a.rows} x {a.rows}, {a.nnz_per_row} distinct columns per row, values U(0,1)"
    return f"R-MAT scale {a.scale}, ef 16, (.57,.19,.19,.05), symmetrised, dedup, no self-loops, values U(0,1)"


def make_workload(a):
    import distspmm_b200 as d
    if a.matrix == "stencil27":
        return d.gen_stencil27(a.grid, seed=a.seed)
    if a.matrix == "uniform":
        return d.gen_uniform(a.rows, a.nnz_per_row, seed=a.seed)
    return d.gen_rmat(a.scale, seed=a.seed)


def config_of(a, world, nnz, M):
    return {"workload": workload_name(a), "matrix": matrix_desc(a),
            "rows": M, "nnz": nnz, "dims": a.dims, "n_rolls": a.n_rolls, "task_dist": a.task_dist,
            "comm_type": a.comm_type, "parallelism": f"row1d_p{world}", "seed": a.seed,
            "partition": a.partition if world > 1 else "single rank", "fetch_scope": a.fetch_scope,
            "pipeline": a.pipeline, "fetch_streams": a.fetch_streams, "selector_platform": a.platform,
            "l2": "flushed between steps (512 MiB write)" if not a.no_flush else "not flushed",
            "b": "U(-1,1) fp32 row-major"}


def host_threads():
    """All host threads this process may run on (torchrun sets OMP_NUM_THREADS=1; the CPU
    arms pass the thread count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(workload):
    """DRAM bytes per launch of the SpMM kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", f"spmm_{workload}.md")
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


class Clocks:
    """nvidia-smi sampling (every 50 ms) kept to the samples taken inside the timed region."""
    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "50"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.5)  # let the sampler come up before the timed region opens
        except OSError:
            self.p = None

    def mark(self, begin: bool):
        if begin:
            self.t0 = datetime.datetime.now()
        else:
            self.t1 = datetime.datetime.now()

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.f.seek(0)
        rows = [r for r in csv.reader(io.StringIO(self.f.read())) if len(r) >= 10]
        os.unlink(self.f.name)

        def inside(r):
            try:
                ts = datetime.datetime.strptime(r[0].strip(), "%Y/%m/%d %H:%M:%S.%f")
            except ValueError:
                return False
            return self.t0 is not None and self.t0 <= ts <= self.t1

        rows = [r for r in rows if inside(r)]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        mx = [float(r[3]) for r in rows if r[3].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[6:10]) if "Active" in v and "Not" not in v})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_spmm_baseline(A, B, budget_s=10.0, max_reps=5):
    """Time the oracle's fp32 OpenMP CSR x dense loop (all host threads) on the full matrix,
    or on a strided row sample when one pass would exceed the budget."""
    import numpy as np

    import oracle
    threads = host_threads()
    C = np.empty((A.num_rows, B.shape[1]), np.float32)
    t0 = time.perf_counter()
    oracle.spmm_f32(A.indptr, A.indices, A.values, B, threads=threads, out=C)
    first = time.perf_counter() - t0
    sample = "full matrix"
    ip, ix, vv, nnz = A.indptr, A.indices, A.values, A.nnz
    if first > budget_s / 2:
        k = int(first / (budget_s / 8)) + 1
        rows = np.arange(0, A.num_rows, k)
        lens = np.diff(A.indptr)[rows]
        ip = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        sel = np.concatenate([np.arange(A.indptr[r], A.indptr[r + 1]) for r in rows])
        ix, vv, nnz = A.indices[sel], A.values[sel], int(ip[-1])
        C = np.empty((rows.size, B.shape[1]), np.float32)
        sample = f"every {k}-th row ({rows.size} rows, {nnz} nnz)"
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_reps and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        oracle.spmm_f32(ip, ix, vv, B, threads=threads, out=C)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(2.0 * nnz * B.shape[1] / t / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{sample}, dims {B.shape[1]}, median of {len(times)} passes"}


def run_reference(a, rank, world):
    """CPU arm: the oracle's fp32 OpenMP loop on rank 0 (other ranks exit without work)."""
    if rank != 0:
        return 0
    import distspmm_b200 as d
    A = make_workload(a)
    B = d.dense_b(A.num_cols, a.dims, seed=a.seed + 1)
    import numpy as np

    import oracle
    threads = host_threads()
    C = np.empty((A.num_rows, a.dims), np.float32)
    t0 = time.perf_counter()
    oracle.spmm_f32(A.indptr, A.indices, A.values, B, threads=threads, out=C)
    one = time.perf_counter() - t0
    # bound the whole run to about two minutes
    k = max(1, int(one * (a.steps + a.warmup) / 120.0) + 1)
    ip, ix, vv, nnz, sample = A.indptr, A.indices, A.values, A.nnz, "full matrix"
    if k > 1:
        rows = np.arange(0, A.num_rows, k)
        lens = np.diff(A.indptr)[rows]
        ip = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        sel = np.concatenate([np.arange(A.indptr[r], A.indptr[r + 1]) for r in rows])
        ix, vv, nnz = A.indices[sel], A.values[sel], int(ip[-1])
        C = np.empty((rows.size, a.dims), np.float32)
        sample = f"every {k}-th row ({rows.size} rows, {nnz} nnz)"
    for _ in range(a.warmup):
        oracle.spmm_f32(ip, ix, vv, B, threads=threads, out=C)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        oracle.spmm_f32(ip, ix, vv, B, threads=threads, out=C)
    dt = (time.perf_counter() - t0) / max(a.steps, 1)
    v = 2.0 * nnz * a.dims / dt / 1e9
    line = {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": config_of(a, 1, A.nnz, A.num_rows),
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{sample}, dims {a.dims}"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    a = parse_args(argv)
    rank, local_rank, world = env_rank()
    if a.impl == "reference":
        return run_reference(a, rank, world)
    import numpy as np
    import torch

    import distspmm_b200 as d
    from distspmm_b200 import planner
    from distspmm_b200.dist import TorchComm, connect_peers, distributed_plan, global_plan, make_rank

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    comm = None
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        # keep stdout to the one JSON line: the NCCL communicator set-up (eager, with
        # device_id) may print a version banner on file descriptor 1; send it to stderr
        with stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            comm = TorchComm()
            comm.barrier()

    # every rank builds the whole matrix (the reference: every rank reads the whole file)
    A = make_workload(a)
    M, nnz = A.num_rows, A.nnz
    lb, ub = planner.bounds(A, world, rank, a.partition)
    local = planner.partition(A, lb, ub)
    if comm is None:
        tiling = planner.tile(local, a.n_rolls)
        plan = global_plan([tiling], a.task_dist, a.n_rolls)
    else:
        tiling, plan = distributed_plan(comm, local, a.n_rolls, a.task_dist)
    R = make_rank(local, rank, world, local_rank, a.dims, M, lb, tiling, plan, a.comm_type, a.platform, a.fetch_streams,
                  fetch_scope=a.fetch_scope, pipeline=a.pipeline)
    if comm is not None:
        connect_peers(comm, R)
    st = R.stats()
    s = torch.cuda.Stream(dev)
    R.fill_b(a.seed + 1, s.cuda_stream)
    torch.cuda.synchronize(dev)
    if comm is not None:
        comm.barrier()
    flush = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def flush_l2():
        if not a.no_flush:
            with torch.cuda.stream(s):
                flush.fill_(1.0)

    # warm-up (untimed)
    for _ in range(a.warmup):
        R.step(s.cuda_stream)
    torch.cuda.synchronize(dev)
    if comm is not None:
        comm.barrier()

    clocks = Clocks(local_rank) if not a.profile else None
    if clocks:
        clocks.start()
    step_ms, compute_ms = [], []
    torch.cuda.synchronize(dev)
    if comm is not None:
        comm.barrier()
    t_wall = time.perf_counter()
    if clocks:
        clocks.mark(True)
    for _ in range(a.steps):
        flush_l2()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        R.step(s.cuda_stream)
        e1.record(s)
        e1.synchronize()
        step_ms.append(e0.elapsed_time(e1))
        compute_ms.append(R.last_compute_ms())
        timeline = R.timeline()
    torch.cuda.synchronize(dev)
    if comm is not None:
        comm.barrier()
    wall = time.perf_counter() - t_wall
    if clocks:
        clocks.mark(False)
    clk = clocks.stop() if clocks else None

    # compute-stream time spent waiting for fetches in the last step (segments not back to back)
    segs = [(t[2], t[3]) for t in timeline if t[2] is not None]
    idle = (segs[-1][1] - segs[0][0]) - sum(e - b for b, e in segs) if segs else 0.0
    idle_max = comm.allreduce_max(idle) if comm is not None else idle
    mean_step = statistics.mean(step_ms)
    mean_compute = statistics.mean(compute_ms)
    if comm is not None:
        t_step = comm.allreduce_max(mean_step)
        t_comp_max = comm.allreduce_max(mean_compute)
    else:
        t_step, t_comp_max = mean_step, mean_compute
    value = 2.0 * nnz * a.dims / (t_step * 1e-3) / 1e9

    # algorithmic HBM bytes of this rank's SpMM (nnz*12 + U*N*4 + m*N*4)
    alg_bytes = st["nnz_local"] * 12 + st["distinct_cols"] * a.dims * 4 + st["m_local"] * a.dims * 4
    peak, peak_kind = measured_peaks()
    achieved = alg_bytes / (mean_compute * 1e-3) / 1e9

    # end to end through the C ABI: pinned host B (owned tiles uploaded), step, C to host
    e2e = None
    if not a.no_e2e and not a.profile:
        Bh = torch.empty((M, a.dims), dtype=torch.float32, pin_memory=True)
        d.dense_b(M, a.dims, a.seed + 1, out=Bh.numpy())
        # Steps back to back as an application runs them: B of step i+1 goes up (H2D
        # stream) while C of step i comes down (D2H stream); each step waits for its B and
        # for the previous C to have left the device, each upload for the previous step's
        # reads of B. On one GPU a second rank object (when memory allows) double-buffers
        # B and C, so the SpMM of step i+1 also overlaps the download of step i. Timed from
        # the first upload to the last download of the K steps.
        slots = [R]
        if comm is None:
            free, _ = torch.cuda.mem_get_info(dev)
            if 4 * (M + (ub - lb)) * a.dims * 4 < free:
                slots.append(make_rank(local, rank, world, local_rank, a.dims, M, lb, tiling, plan, a.comm_type,
                                       a.platform, a.fetch_streams, fetch_scope=a.fetch_scope, pipeline=a.pipeline))
        Chs = [torch.empty((max(ub - lb, 1), a.dims), dtype=torch.float32, pin_memory=True) for _ in slots]
        s_up, s_dn = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def e2e_run(n):
            ev_comp, ev_dn = [None] * len(slots), [None] * len(slots)
            last = None
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(s_up)
            for i in range(n):
                k = i % len(slots)
                X = slots[k]
                if ev_comp[k] is not None:
                    s_up.wait_event(ev_comp[k])  # X's B is free once its previous SpMM is done
                if comm is not None and last is not None:  # ... on every rank: peers read its tiles
                    last.synchronize()
                    comm.barrier()
                X.upload_b_ptr(Bh.data_ptr(), s_up.cuda_stream)
                ev_up = torch.cuda.Event()
                ev_up.record(s_up)
                if comm is not None:  # peers read this rank's tiles only after every upload landed
                    ev_up.synchronize()
                    comm.barrier()
                s.wait_event(ev_up)
                if ev_dn[k] is not None:
                    s.wait_event(ev_dn[k])  # X's C is free once its previous download is done
                X.step(s.cuda_stream)
                ev_comp[k] = last = torch.cuda.Event()
                ev_comp[k].record(s)
                s_dn.wait_event(ev_comp[k])
                if ub > lb:
                    X.download_c_ptr(Chs[k].data_ptr(), s_dn.cuda_stream)
                ev_dn[k] = torch.cuda.Event()
                ev_dn[k].record(s_dn)
            t1.record(s_dn)
            t1.synchronize()
            if comm is not None:
                comm.barrier()
            return t0.elapsed_time(t1) / n

        e2e_run(max(a.warmup, 1))
        n_e2e = max(a.steps, 1)
        t_e2e = e2e_run(n_e2e)
        Ch = Chs[(n_e2e - 1) % len(slots)]
        for X in slots[1:]:
            X.close()
        if comm is not None:
            t_e2e = comm.allreduce_max(t_e2e)
        # spot check of the result against the oracle on a few rows of this rank
        import oracle
        rng = np.random.default_rng(rank)
        rows = rng.choice(ub - lb, size=min(64, ub - lb), replace=False) if ub > lb else np.zeros(0, int)
        lens = np.diff(local.indptr)[rows]
        ip = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
        sel = np.concatenate([np.arange(local.indptr[r], local.indptr[r + 1]) for r in rows]) if rows.size else \
            np.zeros(0, np.int64)
        ref, ab = oracle.spmm_f64(ip, local.indices[sel], local.values[sel], Bh.numpy())
        ok, worst = oracle.check_close(Ch.numpy()[rows], ref, ab, 1e-5)
        if comm is not None:
            worst = comm.allreduce_max(worst)
            ok = worst <= 1.0
        e2e = {"value": round(2.0 * nnz * a.dims / (t_e2e * 1e-3) / 1e9, 3), "unit": UNIT,
               "ms_per_step": round(t_e2e, 4), "h2d_bytes_per_step": st["owned_rows"] * a.dims * 4,
               "d2h_bytes_per_step": (ub - lb) * a.dims * 4,
               "overlap": "H2D of step i+1 with D2H of step i (pinned host buffers, separate streams)"
                          + ("; B and C double-buffered (two rank objects), SpMM overlaps both" if len(slots) > 1 else ""),
               "check": {"rows": int(rows.size), "worst_err_over_tol": round(worst, 4), "ok": bool(ok)}}

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline and not a.profile:
        cpu = cpu_spmm_baseline(A, d.dense_b(M, a.dims, a.seed + 1))

    # Gather stream: every nonzero reads one B row of dims floats through L2 -> L1 (what
    # bounds a gather-per-nonzero kernel, next to the HBM roofline's algorithmic bytes).
    gathered = st["nnz_local"] * a.dims * 4
    gather = {"gathered_bytes_per_launch": gathered, "unit": "GB/s",
              "achieved": round(gathered / (mean_compute * 1e-3) / 1e9, 1)}

    fetch_bytes = st["fetch_bytes"]
    # per rank: nonzeros, rows, phase structure, SpMM time, time waiting for fetches, bytes
    mine = [st["nnz_local"], st["m_local"], st["pipeline"], int(mean_compute * 1e4), int(idle * 1e4),
            st["fetch_bytes"] // 1024]
    per_rank = [mine]
    if comm is not None:
        fetch_bytes = comm.allreduce_sum_i64(fetch_bytes)
        per_rank = [[int(x) for x in r] for r in comm.allgather_i32(np.array(mine, np.int64).clip(max=2**31 - 1))]
    ranks = [{"nnz": r[0], "rows": r[1], "pipeline": ["", "rows", "split"][r[2]], "compute_ms": r[3] / 1e4,
              "idle_ms": r[4] / 1e4, "fetched_kib": r[5]} for r in per_rank]
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(t_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_of(a, world, nnz, M),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": profile_traffic(workload_name(a)),
                     "kernel": "spmm_nnz_kernel / spmm_rows_kernel (+fixup, zero rows)", "rank": rank,
                     "alg_bytes_per_launch": alg_bytes, "launch_ms": round(mean_compute, 4),
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
        "e2e": e2e, "cpu_baseline": cpu, "clocks": clk,
        "gpu_launches": a.steps * st["kernels_per_step"],
        "nvlink": {"fetched_bytes_per_step": fetch_bytes, "pipeline_rank0": ["", "rows", "split"][st["pipeline"]],
                   "phase0_nnz_rank0": st["phase0_nnz"],
                   "max_rank_compute_ms": round(t_comp_max, 4),
                   "max_rank_compute_idle_ms": round(idle_max, 4),
                   "timeline_rank0": timeline if rank == 0 else None, "ranks": ranks},
        "wall_s_timed_region": round(wall, 3),
        "gather": gather,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    R.close()
    if comm is not None:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
