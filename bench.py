#!/usr/bin/env python
"""Benchmark of the distributed CSR x dense SpMM (the hot path of DistSpMM) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...      (one rank per GPU)

Workload (the largest single-GPU one): R-MAT scale 24, edge
factor 16, (a,b,c,d) = (.57,.19,.19,.05), symmetrised, deduplicated, no self-loops
(16,777,216 rows, ~520 M nnz), values U(0,1); dense B 16,777,216 x 128 fp32 U(-1,1);
1-D row partition over the ranks, T = 4 tiles per rank, HSDMA allocation (task_dist 2),
adaptive fetch (comm_type 2). Other configurations are flags (--scale 15/20, --matrix
stencil27 | uniform, --dims). All inputs are seeded synthetic data generated here; at
N > 1 rank 0 writes the matrix once as the reference's binary CSR files (tmpfs) and every
rank reads only its own rows. The matrix is fixed as N grows (strong scaling, as the
reference partitions one matrix).

A step is one distributed SpMM C = A.B over the whole matrix: every rank fetches its
needed remote B rows (copy-engine bulk copies / NVLink gather kernels) and runs its
SpMM segments. Metric: GFLOPS = 2.nnz.dims / t, t = device time of a step (CUDA events
on the launching stream, mean over K steps, max over ranks). L2 is flushed between steps
(a 512 MiB write outside the timed events). `e2e` times the same steps through the C ABI
from pinned host memory: H2D of the rank's owned B tiles, the step, D2H of its C rows,
back to back with B and C double-buffered (two rank objects) so that uploads, SpMM and
downloads of consecutive steps overlap; at N > 1 the ranks order their uploads and
peers' reads with stream-ordered NCCL all-reduces of one element (no host barrier per
step). Every rank then checks a 1 % row sample of its C (plus every hub row) against the
CPU oracle; a failed check makes the run exit non-zero. At N = 1 the line also carries
`cusparse`: the reference's own local SpMM (cuSPARSE per-tile COO, ALG_DEFAULT, beta = 1)
and a whole-matrix CSR cuSPARSE call, timed the same way on the same B.

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
    ap.add_argument("--scale", type=int, default=24, help="R-MAT scale")
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
    ap.add_argument("--pipeline", choices=["auto", "rows", "split", "groups"], default="auto",
                    help="phases: whole rows after their last fetch, nonzeros per ring position, row groups "
                         "fetched group by group, or per matrix")
    ap.add_argument("--groups", type=int, default=0, help="row groups of the groups pipeline (0 = 8)")
    ap.add_argument("--fetch-streams", type=int, default=4, help="concurrent fetch streams (nvlink_num_producers)")
    ap.add_argument("--platform", choices=["h100", "a800", "b200"], default="b200",
                    help="adaptive selector constants (comm_type 2); b200 = the NVLink 5 fit of comm_test")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--csr-cache", default=None,
                    help="directory that keeps generated matrices (binary CSR) for later runs")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-flush", action="store_true")
    ap.add_argument("--no-cusparse", action="store_true", help="skip the cuSPARSE comparison arm (N = 1)")
    ap.add_argument("--no-ref-semantics", action="store_true",
                    help="skip the N > 1 measurement under the reference's partition and merged fetch lists")
    ap.add_argument("--check-frac", type=float, default=0.01, help="fraction of each rank's rows checked")
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


def matrix_key(a):
    """File-name key of the generated matrix (everything that determines it)."""
    if a.matrix == "stencil27":
        return f"stencil{a.grid}_s{a.seed}"
    if a.matrix == "uniform":
        return f"uniform{a.rows}x{a.nnz_per_row}_s{a.seed}"
    return f"rmat{a.scale}_s{a.seed}"


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
            "pipeline": a.pipeline, "groups": a.groups or 8, "fetch_streams": a.fetch_streams, "selector_platform": a.platform,
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




def hub_degree(a):
    """Rows longer than this are always checked (R-MAT hubs, cut into pieces by the kernels)."""
    return max(4096, 1 << max(0, a.scale - 10)) if a.matrix == "rmat" else 1 << 30


def row_sample(indptr, target_nnz, offset=0):
    """Every k-th row, k chosen so that the sample holds about target_nnz nonzeros, as a
    compact CSR (indptr rebased) plus the sampled row ids."""
    import numpy as np
    m = indptr.size - 1
    nnz = int(indptr[-1] - indptr[0])
    k = max(1, -(-nnz // max(target_nnz, 1)))
    rows = np.arange(offset % k, m, k, dtype=np.int64)
    lens = indptr[rows + 1] - indptr[rows]
    ip = np.zeros(rows.size + 1, np.int64)
    np.cumsum(lens, out=ip[1:])
    starts = np.repeat(indptr[rows] - ip[:-1], lens)
    sel = np.arange(int(ip[-1]), dtype=np.int64) + starts
    return k, rows, ip, sel


def compact_b(cols, dims, seed):
    """B rows of the distinct columns `cols` needs, and cols renumbered into them."""
    import numpy as np

    import distspmm_b200 as d
    uniq, inv = np.unique(cols, return_inverse=True)
    return d.dense_b_rows(uniq, dims, seed), inv.astype(np.int64)


def cpu_spmm_baseline(A, dims, seed, budget_s=10.0, max_reps=5, target_nnz=16 << 20):
    """Time the oracle's fp32 OpenMP CSR x dense loop (all host threads) on a strided row
    sample of about target_nnz nonzeros (the whole matrix when it is smaller)."""
    import numpy as np

    import oracle
    threads = host_threads()
    k, rows, ip, sel = row_sample(A.indptr, target_nnz)
    Bc, cols = compact_b(A.indices[sel], dims, seed)
    vals = A.values[sel]
    nnz = int(ip[-1])
    C = np.empty((rows.size, dims), np.float32)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_reps and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        oracle.spmm_f32(ip, cols, vals, Bc, threads=threads, out=C)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    sample = "full matrix" if k == 1 else f"every {k}-th row ({rows.size} rows, {nnz} nnz)"
    return {"value": round(2.0 * nnz * dims / t / 1e9, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{sample}, dims {dims}, B rows of the sampled columns, median of {len(times)} passes"}


def run_reference(a, rank, world):
    """CPU arm: the oracle's fp32 OpenMP loop on rank 0 (other ranks exit without work),
    each step one pass over a strided row sample of the workload (about 8 M nonzeros)."""
    if rank != 0:
        return 0
    import numpy as np

    import oracle
    A = make_workload(a)
    threads = host_threads()
    k, rows, ip, sel = row_sample(A.indptr, 8 << 20)
    Bc, cols = compact_b(A.indices[sel], a.dims, a.seed + 1)
    vals = A.values[sel]
    nnz = int(ip[-1])
    C = np.empty((rows.size, a.dims), np.float32)
    for _ in range(a.warmup):
        oracle.spmm_f32(ip, cols, vals, Bc, threads=threads, out=C)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        oracle.spmm_f32(ip, cols, vals, Bc, threads=threads, out=C)
    dt = (time.perf_counter() - t0) / max(a.steps, 1)
    v = 2.0 * nnz * a.dims / dt / 1e9
    sample = "full matrix" if k == 1 else f"every {k}-th row ({rows.size} rows, {nnz} nnz)"
    line = {"metric": METRIC, "value": round(v, 3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": config_of(a, 1, A.nnz, A.num_rows),
            "cpu_baseline": {"value": round(v, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{sample}, dims {a.dims}"},
            "e2e": {"value": round(v, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def load_local(a, rank, world, comm):
    """This rank's rows. N = 1: the generated matrix itself. N > 1: rank 0 generates the
    matrix once and writes the reference's binary CSR files to tmpfs; every rank reads the
    row pointer, finds its rows (planner.bounds) and reads only those (load_rows).
    Returns (local, M, nnz, lb, ub, cleanup, rows_for): rows_for(partition) reads this
    rank's rows under another partition (N > 1; None at N = 1)."""
    import numpy as np

    import distspmm_b200 as d
    from distspmm_b200 import planner
    # --csr-cache DIR: the generated matrix is kept in DIR/<matrix key> (reference binary CSR
    # files) and read back by later runs with the same matrix arguments
    key = os.path.join(a.csr_cache, f"{matrix_key(a)}") if a.csr_cache else None
    cached = key is not None and os.path.exists(os.path.join(key, "A_indptr.bin"))

    def generate_into(dirpath):
        A = make_workload(a)
        tmpd = tempfile.mkdtemp(prefix=".dsp_tmp_", dir=os.path.dirname(dirpath))
        d.save_csr(os.path.join(tmpd, "A"), A)
        try:
            os.rename(tmpd, dirpath)
        except OSError:  # another run stored it first
            for f in os.listdir(tmpd):
                os.unlink(os.path.join(tmpd, f))
            os.rmdir(tmpd)
        return A

    if world == 1:
        if cached:
            ip = np.fromfile(os.path.join(key, "A_indptr.bin"), np.int64)
            A = d.load_rows(os.path.join(key, "A"), 0, ip.size - 1)
        elif key is not None:
            os.makedirs(a.csr_cache, exist_ok=True)
            A = generate_into(key)
        else:
            A = make_workload(a)
        return A, A.num_rows, A.nnz, 0, A.num_rows, None, None
    import torch.distributed as dist
    box = [None]
    if rank == 0:
        if cached:
            tmp = key
        elif key is not None:
            os.makedirs(a.csr_cache, exist_ok=True)
            generate_into(key)
            tmp = key
        else:
            A = make_workload(a)
            base = "/dev/shm" if os.path.isdir("/dev/shm") else None
            tmp = tempfile.mkdtemp(prefix="dsp_bench_", dir=base)
            d.save_csr(os.path.join(tmp, "A"), A)
            del A
        box[0] = tmp
    dist.broadcast_object_list(box, src=0)
    tmp = box[0]
    prefix = os.path.join(tmp, "A")
    ip = np.fromfile(prefix + "_indptr.bin", np.int64)
    M = ip.size - 1
    nnz = int(ip[-1])
    g = d.Csr(ip, np.zeros(0, np.int64), np.zeros(0, np.float32), M, M)
    lb, ub = planner.bounds(g, world, rank, a.partition)
    local = d.load_rows(prefix, lb, ub)
    comm.barrier()  # every rank has read its rows

    def cleanup():
        if rank == 0 and key is None:
            for f in os.listdir(tmp):
                os.unlink(os.path.join(tmp, f))
            os.rmdir(tmp)

    def rows_for(partition):
        lb2, ub2 = planner.bounds(g, world, rank, partition)
        return d.load_rows(prefix, lb2, ub2), lb2, ub2
    return local, M, nnz, lb, ub, cleanup, rows_for


def check_c(a, local, C_rows_of, rank):
    """Sampled check of this rank's C against the oracle: every k-th local row (k from
    --check-frac, offset by the rank) plus every row longer than hub_degree(a). C_rows_of
    maps local row ids to their computed rows. Returns (rows checked, worst ratio)."""
    import distspmm_b200 as d
    import oracle
    rows = oracle.sample_rows(local.num_rows, a.check_frac, local.indptr, hub_degree(a), offset=rank)
    if rows.size == 0:
        return 0, 0.0
    got = C_rows_of(rows)
    _, worst = oracle.check_rows(local.indptr, local.indices, local.values,
                                 lambda cols: d.dense_b_rows(cols, a.dims, a.seed + 1), rows, got, 1e-5)
    return int(rows.size), float(worst)


def cusparse_arm(a, local, M, R, flush_l2, ours_ms):
    """The reference's local SpMM on this GPU, on R's B: cuSPARSE per-tile COO (int64,
    ALG_DEFAULT, beta = 1 over T = n_rolls tiles; src/dist_spmm_node.cu:206-234, :354-385)
    and a whole-matrix CSR call; CUDA events, L2 flushed before each run, mean of 5."""
    import torch

    import baseline
    dev = torch.device("cuda", torch.cuda.current_device())
    C = torch.empty((local.num_rows, a.dims), dtype=torch.float32, device=dev)
    s = torch.cuda.Stream(dev)
    arm = baseline.CusparseArm(local, M, a.n_rolls, a.dims, R.b_ptr(), C.data_ptr())

    def timed(fn, pre=None, reps=5):
        fn()
        torch.cuda.synchronize(dev)
        ts = []
        for _ in range(reps):
            flush_l2()
            if pre:
                with torch.cuda.stream(s):
                    pre()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            fn()
            e1.record(s)
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.mean(ts)

    zero = lambda: C.zero_()  # noqa: E731 — the reference zeroes C before each rep, untimed
    t_tiles = timed(lambda: arm.run_tiles(R.b_ptr(), C.data_ptr(), s.cuda_stream), pre=zero)
    _, w_tiles = check_c(a, local, lambda r: C[torch.from_numpy(r).to(dev)].cpu().numpy(), 0)
    t_csr = timed(lambda: arm.run_csr(R.b_ptr(), C.data_ptr(), s.cuda_stream))
    _, w_csr = check_c(a, local, lambda r: C[torch.from_numpy(r).to(dev)].cpu().numpy(), 0)
    arm.close()
    del C
    torch.cuda.empty_cache()
    g = lambda ms: round(2.0 * local.nnz * a.dims / (ms * 1e-3) / 1e9, 3)  # noqa: E731
    best = min(t_tiles, t_csr)
    return {"reference_tiles_coo": {"ms": round(t_tiles, 4), "gflops": g(t_tiles), "tiles": a.n_rolls,
                                    "check_worst_err_over_tol": round(w_tiles, 4)},
            "csr_whole_matrix": {"ms": round(t_csr, 4), "gflops": g(t_csr),
                                 "check_worst_err_over_tol": round(w_csr, 4)},
            "ours_ms": round(ours_ms, 4), "speedup_vs_best_cusparse": round(best / ours_ms, 3),
            "how": "cusparseSpMM fp32, int64 indices, CUSPARSE_SPMM_ALG_DEFAULT; descriptors and buffers made "
                   "once; CUDA events, L2 flushed before each of 5 runs; same B as ours"}


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
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
            comm = TorchComm()
            comm.barrier()

    t_setup = time.perf_counter()
    local, M, nnz, lb, ub, cleanup, rows_for = load_local(a, rank, world, comm)
    t_loaded = time.perf_counter()
    if comm is None:
        tiling = planner.tile(local, a.n_rolls)
        plan = global_plan([tiling], a.task_dist, a.n_rolls)
    else:
        tiling, plan = distributed_plan(comm, local, a.n_rolls, a.task_dist)
    t_planned = time.perf_counter()

    def new_rank():
        X = make_rank(local, rank, world, local_rank, a.dims, M, lb, tiling, plan, a.comm_type, a.platform,
                      a.fetch_streams, fetch_scope=a.fetch_scope, pipeline=a.pipeline, groups=a.groups)
        if comm is not None:
            connect_peers(comm, X)
        return X

    R = new_rank()
    st = R.stats()
    s = torch.cuda.Stream(dev)
    R.fill_b(a.seed + 1, s.cuda_stream)
    torch.cuda.synchronize(dev)
    if comm is not None:
        comm.barrier()
    setup_s = time.perf_counter() - t_setup
    # where set-up goes: matrix generation / reading, tiling + allocation + lists, the
    # rank's device operands and fetch plan (with B filled)
    setup_parts = {"load_s": round(t_loaded - t_setup, 1), "plan_s": round(t_planned - t_loaded, 1),
                   "rank_s": round(setup_s - (t_planned - t_setup), 1)}
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
    R.check_error()

    # the result of the timed steps, checked before anything else runs
    if ub > lb:
        torch.cuda.synchronize(dev)
        Ch0 = np.empty((ub - lb, a.dims), np.float32)
        R.download_c(Ch0)
        torch.cuda.synchronize(dev)
        n_dev, worst_dev = check_c(a, local, lambda r: Ch0[r], rank)
        del Ch0
    else:
        n_dev, worst_dev = 0, 0.0

    # compute-stream time spent waiting for fetches in the last step: from the step's start
    # (timeline origin) to the last segment's end, minus the segments' own durations, so a
    # wait before the first segment (an empty owned phase) counts too
    segs = [(t[2], t[3]) for t in timeline if t[2] is not None]
    idle = max(0.0, segs[-1][1] - sum(e - b for b, e in segs)) if segs else 0.0
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

    # end to end through the C ABI: pinned host B (the rank's owned tiles), step, C to host
    e2e = None
    n_e2e_chk, worst_e2e = 0, 0.0
    if not a.no_e2e and not a.profile:
        owned = R.owned_tiles()
        n_owned = sum(n for _, n in owned)
        Bh = torch.empty((max(n_owned, 1), a.dims), dtype=torch.float32, pin_memory=True)
        o = 0
        for row0, n in owned:
            d.dense_b(n, a.dims, a.seed + 1, row0=row0, out=Bh.numpy()[o:o + n])
            o += n
        # Steps back to back as an application runs them, B and C double-buffered (a second
        # rank object when memory allows): step i+1's upload (H2D stream) overlaps step i's
        # SpMM and step i's download (D2H stream) overlaps step i+1's SpMM. Each upload waits
        # until no rank reads that slot's B any more, each step until every rank's upload
        # of its slot landed: with N > 1 both conditions are stream-ordered one-element NCCL
        # all-reduces on a sync stream, so the host never blocks between steps.
        slots = [R]
        free, _ = torch.cuda.mem_get_info(dev)
        room = 1.0 if st["device_bytes"] + (1 << 30) < free else 0.0
        if comm is not None:  # the same choice on every rank (a second slot means collectives)
            room = -comm.allreduce_max(-room)
        if room > 0:
            slots.append(new_rank())
        Chs = [torch.empty((max(ub - lb, 1), a.dims), dtype=torch.float32, pin_memory=True) for _ in slots]
        s_up, s_dn, s_sync = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        tok = torch.zeros(1, dtype=torch.float32, device=dev)

        def global_event(ev):
            """An event that completes once `ev` completed on every rank."""
            if comm is None:
                return ev
            s_sync.wait_event(ev)
            with torch.cuda.stream(s_sync):
                comm.dist.all_reduce(tok, group=comm.group)
            g = torch.cuda.Event()
            g.record(s_sync)
            return g

        def e2e_run(n):
            ev_free, ev_dn = [None] * len(slots), [None] * len(slots)
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record(s_up)
            for i in range(n):
                k = i % len(slots)
                X = slots[k]
                if ev_free[k] is not None:
                    s_up.wait_event(ev_free[k])  # no rank reads X's B any more
                X.upload_b_owned_ptr(Bh.data_ptr(), s_up.cuda_stream)
                ev_up = torch.cuda.Event()
                ev_up.record(s_up)
                s.wait_event(global_event(ev_up))  # every rank's owned tiles of this step landed
                if ev_dn[k] is not None:
                    s.wait_event(ev_dn[k])  # X's C is free once its previous download is done
                X.step(s.cuda_stream)
                ev_comp = torch.cuda.Event()
                ev_comp.record(s)
                ev_free[k] = global_event(ev_comp)
                s_dn.wait_event(ev_comp)
                if ub > lb:
                    X.download_c_ptr(Chs[k].data_ptr(), s_dn.cuda_stream)
                ev_dn[k] = torch.cuda.Event()
                ev_dn[k].record(s_dn)
            t1.record(s_dn)
            t1.synchronize()
            torch.cuda.synchronize(dev)
            return t0.elapsed_time(t1) / n

        e2e_run(max(a.warmup, 1))
        n_e2e = max(a.steps, 1)
        t_e2e = e2e_run(n_e2e)
        Ch = Chs[(n_e2e - 1) % len(slots)]
        for X in slots:
            X.check_error()
        for X in slots[1:]:
            X.close()
        if comm is not None:
            comm.barrier()
            t_e2e = comm.allreduce_max(t_e2e)
        if ub > lb:
            n_e2e_chk, worst_e2e = check_c(a, local, lambda r: Ch.numpy()[r], rank)
        e2e = {"value": round(2.0 * nnz * a.dims / (t_e2e * 1e-3) / 1e9, 3), "unit": UNIT,
               "ms_per_step": round(t_e2e, 4), "h2d_bytes_per_step": n_owned * a.dims * 4,
               "d2h_bytes_per_step": (ub - lb) * a.dims * 4,
               "overlap": "B and C double-buffered (two rank objects)" if len(slots) > 1 else "single buffer",
               "sync": "stream-ordered one-element NCCL all-reduces" if comm is not None else "events"}
        del Bh, Chs

    # correctness of this rank's rows (device-timed steps and the e2e steps), all ranks
    worst = max(worst_dev, worst_e2e)
    n_chk = n_dev + n_e2e_chk
    if comm is not None:
        worst = comm.allreduce_max(worst)
        n_chk = comm.allreduce_sum_i64(n_chk)
    check = {"rows_checked_all_ranks": n_chk, "frac_per_rank": a.check_frac,
             "plus_rows_longer_than": hub_degree(a), "worst_err_over_tol": round(worst, 4), "ok": bool(worst <= 1.0),
             "tolerance": "|dC| <= 1e-5 * (|A|.|B|) elementwise vs the double-accumulated CPU oracle"}

    cpu = None
    cus = None
    if world == 1 and not a.profile:
        if not a.no_cusparse:
            try:
                cus = cusparse_arm(a, local, M, R, flush_l2, mean_compute)
            except Exception as e:  # noqa: BLE001 — a comparison arm must not sink the line
                cus = {"error": str(e)[:300]}
        if not a.no_cpu_baseline:
            cpu = cpu_spmm_baseline(local, a.dims, a.seed + 1)

    # Gather stream: every nonzero reads one B row of dims floats through L2 -> L1 (what
    # bounds a gather-per-nonzero kernel, next to the HBM roofline's algorithmic bytes).
    gathered = st["nnz_local"] * a.dims * 4
    gather = {"gathered_bytes_per_launch": gathered, "unit": "GB/s",
              "achieved": round(gathered / (mean_compute * 1e-3) / 1e9, 1)}

    fetch_bytes = st["fetch_bytes"]
    # per rank: nonzeros, rows, phase structure, SpMM time, time waiting for fetches, bytes
    mine = [st["nnz_local"], st["m_local"], st["pipeline"], int(mean_compute * 1e4), int(idle * 1e4),
            st["fetch_bytes"] // 1024, int(st["model_rows_ms"] * 1e4), int(st["model_split_ms"] * 1e4),
            int(st["model_groups_ms"] * 1e4)]
    per_rank = [mine]
    if comm is not None:
        fetch_bytes = comm.allreduce_sum_i64(fetch_bytes)
        per_rank = [[int(x) for x in r] for r in comm.allgather_i32(np.array(mine, np.int64).clip(max=2**31 - 1))]
    ranks = [{"nnz": r[0], "rows": r[1], "pipeline": ["", "rows", "split", "groups"][r[2]], "compute_ms": r[3] / 1e4,
              "idle_ms": r[4] / 1e4, "fetched_kib": r[5],
              "auto_model_ms": {"rows": r[6] / 1e4, "split": r[7] / 1e4, "groups": r[8] / 1e4}} for r in per_rank]
    traffic = profile_traffic(workload_name(a)) if world == 1 else None
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(t_step, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config_of(a, world, nnz, M),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": "the rank's SpMM phases: spmm_warp_kernel (nnz-split) / spmm_dia_kernel (banded) / spmm_rows_kernel, + fixup and zero rows", "rank": rank,
                     "alg_bytes_per_launch": alg_bytes, "launch_ms": round(mean_compute, 4),
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
        "e2e": e2e, "cpu_baseline": cpu, "cusparse": cus, "check": check, "clocks": clk,
        "gpu_launches": a.steps * st["kernels_per_step"],
        "nvlink": {"fetched_bytes_per_step": fetch_bytes, "pipeline_rank0": ["", "rows", "split", "groups"][st["pipeline"]],
                   "phase0_nnz_rank0": st["phase0_nnz"],
                   "max_rank_compute_ms": round(t_comp_max, 4),
                   "max_rank_compute_idle_ms": round(idle_max, 4),
                   "timeline_rank0": timeline if rank == 0 else None, "ranks": ranks},
        "wall_s_timed_region": round(wall, 3), "setup_s": round(setup_s, 1), "setup_parts": setup_parts,
        "gather": gather,
    }
    R.close()
    # N > 1: the reference's own data movement on the same matrix — equal-row partition
    # (src/dist_spmm_node.cu:85-93), node-merged fetch lists (src/utils.h:439-547) and its
    # per-tile accumulation in ring order (the split pipeline, :329-394) — timed the same
    # way, labelled beside the line's own (work-balanced rows, per-rank lists, AUTO pipeline)
    if comm is not None and not a.profile and not a.no_ref_semantics:
        local2, lb2, ub2 = rows_for("rows")
        tiling2, plan2 = distributed_plan(comm, local2, a.n_rolls, a.task_dist)
        R2 = make_rank(local2, rank, world, local_rank, a.dims, M, lb2, tiling2, plan2, a.comm_type, a.platform,
                       a.fetch_streams, fetch_scope="node", pipeline="split")
        connect_peers(comm, R2)
        R2.fill_b(a.seed + 1, s.cuda_stream)
        torch.cuda.synchronize(dev)
        comm.barrier()
        for _ in range(a.warmup):
            R2.step(s.cuda_stream)
        torch.cuda.synchronize(dev)
        comm.barrier()
        ms2 = []
        for _ in range(a.steps):
            flush_l2()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            R2.step(s.cuda_stream)
            e1.record(s)
            e1.synchronize()
            ms2.append(e0.elapsed_time(e1))
        torch.cuda.synchronize(dev)
        comm.barrier()
        R2.check_error()
        st2 = R2.stats()
        t2 = comm.allreduce_max(statistics.mean(ms2))
        f2 = comm.allreduce_sum_i64(st2["fetch_bytes"])
        nnz_max = comm.allreduce_max(float(st2["nnz_local"]))
        R2.close()
        line["reference_semantics"] = {
            "partition": "rows (ceil(M/P) rows per rank)", "fetch_scope": "node (merged lists)",
            "pipeline": "split (per ring position, rows accumulated)",
            "value": round(2.0 * nnz * a.dims / (t2 * 1e-3) / 1e9, 3), "unit": UNIT, "ms_per_step": round(t2, 4),
            "fetched_bytes_per_step": f2, "max_rank_nnz": int(nnz_max),
            "pipeline_rank0": ["", "rows", "split", "groups"][st2["pipeline"]]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.barrier()
        if cleanup:
            cleanup()
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0 if check["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
