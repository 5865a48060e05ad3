"""Multi-rank pipeline parity on the GPU(s) available: P ranks in one process (sharing a
GPU when there is only one), each fetching remote B rows from its peers' buffers and
writing each C row once, in the phase after the last fetch it depends on; the gathered C
must match the oracle. Remote rows are
poisoned with NaN before the step, so a row that was not fetched (or fetched after its
use) makes C non-finite instead of passing silently."""
import os
import subprocess

import numpy as np
import pytest

import distspmm_b200 as d
import oracle
from distspmm_b200 import planner

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _devices(world):
    import torch
    n = torch.cuda.device_count()
    return [p % n for p in range(world)]


def _run_group(A, world, dims, rolls, task_dist, comm_type, seed=21, poison=True, fetch_engine="lsu",
               partition="rows", fetch_scope="node", pipeline="auto", groups=0):
    import torch
    from distspmm_b200.dist import build_local_group
    g = build_local_group(A, world, _devices(world), dims, rolls, task_dist, comm_type, fetch_engine=fetch_engine,
                          partition=partition, fetch_scope=fetch_scope, pipeline=pipeline, groups=groups)
    for r in g.ranks:
        if poison:
            r.poison_remote()
        r.fill_b(seed)
    for dev in set(_devices(world)):
        torch.cuda.synchronize(dev)
    g.step()
    for dev in set(_devices(world)):
        torch.cuda.synchronize(dev)
    for r in g.ranks:
        r.check_error()  # no fetch wait gave up
    C = np.zeros((A.num_rows, dims), np.float32)
    for r, (lb, ub) in zip(g.ranks, g.bounds):
        if ub > lb:
            part = np.empty((ub - lb, dims), np.float32)
            r.download_c(part)
            torch.cuda.synchronize(r.device)
            C[lb:ub] = part
    return g, C


def _check(A, C, dims, seed=21):
    B = d.dense_b(A.num_cols, dims, seed)
    ref, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    assert np.isfinite(C).all(), "a remote row was used before it was fetched"
    ok, worst = oracle.check_close(C, ref, ab, RTOL)
    assert ok, worst


@pytest.fixture(scope="module")
def rmat12():
    return d.gen_rmat(12, seed=8)


@pytest.mark.parametrize("world,rolls,task_dist,comm_type", [
    (2, 4, 2, 2), (2, 1, 0, 0), (2, 2, 0, 1), (4, 4, 2, 2), (4, 2, 1, 0), (8, 4, 2, 2), (8, 4, 0, 1),
    (3, 3, 2, 2),
])
def test_group_parity_rmat(gpu, rmat12, world, rolls, task_dist, comm_type):
    g, C = _run_group(rmat12, world, 128, rolls, task_dist, comm_type)
    _check(rmat12, C, 128)
    st = [r.stats() for r in g.ranks]
    if comm_type == 0:
        assert all(s["fetch_sparse_tiles"] == 0 for s in st)
    if comm_type == 1:
        assert all(s["fetch_bulk_tiles"] == 0 for s in st)
    # fetched rows: sparse tiles move the merged needed lists, bulk tiles whole slices
    for p, (r, s) in enumerate(zip(g.ranks, st)):
        exp = 0
        for t in range(g.plan.T):
            if g.plan.remap[t] == p or g.tilings[p].nnz[t] == 0:
                continue
            exp += g.plan.n_col[t] if r.sparse[t] else g.tilings[p].n_slice[t]
        assert s["fetch_rows"] == exp
    g.close()


@pytest.mark.parametrize("engine", ["lsu", "tma"])
@pytest.mark.parametrize("dims", [4, 128, 100, 1024])
def test_group_parity_fetch_engines(gpu, rmat12, engine, dims):
    """Both sparse-fetch engines (TMA needs 16-byte rows; dims = 100 and other odd widths use
    the vector or scalar gather instead)."""
    g, C = _run_group(rmat12, 4, dims, 2, 2, 1, fetch_engine=engine)
    _check(rmat12, C, dims)
    assert all(r.stats()["fetch_sparse_tiles"] > 0 for r in g.ranks)
    g.close()


@pytest.mark.parametrize("dims", [32, 100, 256])
def test_group_parity_widths(gpu, rmat12, dims):
    g, C = _run_group(rmat12, 4, dims, 2, 2, 2)
    _check(rmat12, C, dims)
    g.close()


def test_group_stencil_and_uniform(gpu):
    for A in (d.gen_stencil27(14, seed=2), d.gen_uniform(4096, 16, seed=3)):
        g, C = _run_group(A, 4, 64, 4, 2, 2)
        _check(A, C, 64)
        g.close()


def test_group_upload_from_host_and_repeat(gpu, rmat12):
    """The e2e path: owned tiles uploaded from a host B, several steps in a row."""
    import torch
    from distspmm_b200.dist import build_local_group
    dims = 64
    g = build_local_group(rmat12, 2, _devices(2), dims, 4, 2, 2)
    Bh = d.dense_b(rmat12.num_cols, dims, seed=99)
    for it in range(3):
        for r in g.ranks:
            r.upload_b(Bh)
        for dev in set(_devices(2)):
            torch.cuda.synchronize(dev)
        g.step()
    C = np.zeros((rmat12.num_rows, dims), np.float32)
    for r, (lb, ub) in zip(g.ranks, g.bounds):
        part = np.empty((ub - lb, dims), np.float32)
        r.download_c(part)
        torch.cuda.synchronize(r.device)
        C[lb:ub] = part
    _check(rmat12, C, dims, seed=99)
    g.close()


@pytest.mark.parametrize("partition,fetch_scope", [("balanced", "node"), ("rows", "rank"), ("balanced", "rank")])
@pytest.mark.parametrize("world,comm_type", [(2, 2), (3, 1), (4, 0), (8, 2)])
def test_group_parity_partition_and_fetch_scope(gpu, rmat12, partition, fetch_scope, world, comm_type):
    """Work-balanced rows and per-rank fetch lists: same C (remote rows NaN-poisoned, so a
    row missing from a rank's own list would show), fewer fetched rows per rank."""
    g, C = _run_group(rmat12, world, 128, 4, 2, comm_type, partition=partition, fetch_scope=fetch_scope)
    _check(rmat12, C, 128)
    if partition == "balanced":
        cost = [int(rmat12.indptr[ub] - rmat12.indptr[lb]) + (ub - lb) for lb, ub in g.bounds]
        assert max(cost) <= (rmat12.nnz + rmat12.num_rows) / world + int(np.diff(rmat12.indptr).max()) + 1
    if fetch_scope == "rank" and comm_type == 1:  # all sparse: each rank fetches only its own rows
        for r, t in zip(g.ranks, g.tilings):
            remote = sum(int(t.n_col[k]) for k in range(g.plan.T)
                         if g.plan.remap[k] != r.rank and t.nnz[k] > 0)
            assert r.stats()["fetch_rows"] == remote
    g.close()


@pytest.mark.parametrize("pipeline", ["rows", "split"])
@pytest.mark.parametrize("world,comm_type,partition", [(2, 2, "rows"), (3, 1, "balanced"), (4, 0, "balanced"),
                                                       (8, 2, "balanced")])
def test_group_parity_pipelines(gpu, rmat12, pipeline, world, comm_type, partition):
    """Both phase structures give the oracle's C: whole rows after their last fetch, or
    nonzeros per ring position with rows written by their first phase and accumulated by
    later ones (remote rows NaN-poisoned before the step)."""
    g, C = _run_group(rmat12, world, 128, 4, 2, comm_type, partition=partition, fetch_scope="rank",
                      pipeline=pipeline)
    _check(rmat12, C, 128)
    assert all(r.stats()["pipeline"] == (1 if pipeline == "rows" else 2) for r in g.ranks)
    g.close()


@pytest.mark.parametrize("world,comm_type,partition,groups", [
    (2, 2, "rows", 0), (3, 1, "balanced", 3), (4, 0, "balanced", 8), (8, 2, "balanced", 8), (8, 1, "rows", 1),
    (2, 1, "balanced", 5000)])
def test_group_parity_row_groups(gpu, rmat12, world, comm_type, partition, groups):
    """Row groups: the owned-column nonzeros of every row run first, then each group's remote
    nonzeros (added to the rows the first segment wrote); every remote row arrives with the
    first group that needs it and each group waits only for its own and earlier groups'
    fetches (remote rows NaN-poisoned before the step, so a row used before it landed shows
    up). Includes one group, more groups than the byte-sized segment ids allow, and
    bulk-only fetches."""
    g, C = _run_group(rmat12, world, 128, 4, 2, comm_type, partition=partition, fetch_scope="rank",
                      pipeline="groups", groups=groups)
    _check(rmat12, C, 128)
    for r in g.ranks:
        st = r.stats()
        assert st["pipeline"] == 3
        G = min(groups or 8, max(st["m_local"], 1), 253)
        assert st["timeline_len"] == max(world, G + 1)  # segment 0 (owned columns) + one per group
        tl = r.timeline()
        # a group's SpMM starts after the fetch kernels it depends on were issued: groups
        # run in order on the compute stream
        segs = [t for t in tl if t[2] is not None]
        assert all(a[3] <= b[2] + 1e-3 for a, b in zip(segs, segs[1:]))
    g.close()


def test_group_row_groups_stencil_and_widths(gpu):
    A = d.gen_stencil27(16, seed=9)
    for dims in (64, 128, 256):
        g, C = _run_group(A, 4, dims, 2, 2, 2, partition="balanced", fetch_scope="rank", pipeline="groups")
        _check(A, C, dims)
        g.close()


@pytest.mark.parametrize("dims", [4, 100, 256])
def test_group_split_pipeline_widths(gpu, rmat12, dims):
    g, C = _run_group(rmat12, 4, dims, 2, 2, 2, pipeline="split")
    _check(rmat12, C, dims)
    g.close()


def _auto_pipeline(g, p, A, dims):
    """The AUTO rule restated: whole rows (1) when the rows needing only owned tiles hold at
    least half the nonzeros; otherwise the modelled step time of rows (1), split (2) and row
    groups (3) per rank — a nonzero one B-row gather at 10 TB/s, a fetched row over NVLink at
    730 GB/s, an accumulated piece two gathers, a group segment 60 us — with rows kept
    unless the best other is >= 3 % shorter."""
    lb, ub = g.bounds[p]
    ip = np.asarray(A.indptr[lb:ub + 1]) - A.indptr[lb]
    cols = np.asarray(A.indices[A.indptr[lb]:A.indptr[ub]])
    P = len(g.ranks)
    pos = (g.plan.remap[cols // g.plan.cpt] - p) % P
    m = ub - lb
    rowid = np.repeat(np.arange(m), np.diff(ip))
    last = np.full(m, -1)
    np.maximum.at(last, rowid, pos)
    phase0 = int(np.diff(ip)[last == 0].sum())
    local = int((pos == 0).sum())
    nnz = int(ip[-1])
    if 2 * phase0 >= nnz:
        return 1
    first = np.full(m, P)
    np.minimum.at(first, rowid, pos)
    touched = np.zeros(m, np.int64)
    np.add.at(touched, np.unique(rowid.astype(np.int64) * P + pos) // P, 1)
    acc_pieces = int(np.maximum(touched - 1, 0).sum())
    group_pieces = int(((touched > 1) & (first == 0)).sum())
    fetch_rows = g.ranks[p].stats()["fetch_rows"]
    G = max(1, min(8, max(m, 1), 253))
    t_nnz, t_fetch = dims * 4.0 / 10e12, fetch_rows * dims * 4.0 / 730e9
    t_all, t_p0, t_loc = nnz * t_nnz, phase0 * t_nnz, local * t_nnz
    rows = max(t_fetch, t_p0) + (t_all - t_p0)
    split = max(t_fetch, t_loc) + (t_all - t_loc) + 2.0 * acc_pieces * t_nnz
    groups = max(t_fetch + (t_all - t_loc) / G, t_all) + 2.0 * group_pieces * t_nnz + G * 60e-6
    if min(split, groups) < 0.97 * rows:
        return 2 if split <= groups else 3
    return 1


def test_pipeline_auto_choice(gpu, rmat12):
    """AUTO follows its rule on R-MAT; a stencil stays on whole rows (most rows need only
    owned tiles); a uniform matrix on 2 ranks splits (half of every row local, every row
    needing the peer)."""
    from distspmm_b200.dist import build_local_group
    g = build_local_group(rmat12, 4, _devices(4), 64, 4, 2, 2, partition="balanced", fetch_scope="rank")
    assert [r.stats()["pipeline"] for r in g.ranks] == [_auto_pipeline(g, p, rmat12, 64) for p in range(4)]
    g.close()
    U = d.gen_uniform(4096, 32, seed=3)
    g = build_local_group(U, 2, _devices(2), 64, 4, 2, 2, partition="balanced", fetch_scope="rank")
    assert [r.stats()["pipeline"] for r in g.ranks] == [2] * 2
    g.close()
    A = d.gen_stencil27(20, seed=4)
    g = build_local_group(A, 4, _devices(4), 64, 4, 2, 2, partition="balanced", fetch_scope="rank")
    assert [r.stats()["pipeline"] for r in g.ranks] == [1] * 4
    g.close()


def test_group_stencil_per_rank_fetch(gpu):
    A = d.gen_stencil27(20, seed=4)
    g, C = _run_group(A, 4, 128, 4, 2, 2, partition="balanced", fetch_scope="rank")
    _check(A, C, 128)
    g.close()


def test_dsp_run_pipeline(gpu, rmat12):
    """dsp_run: the whole dist_spmm_node program in-process, C returned to the host."""
    import ctypes
    from distspmm_b200 import _lib
    world, dims = 4, 128
    devs = (ctypes.c_int * world)(*_devices(world))
    C = np.zeros((rmat12.num_rows, dims), np.float32)
    c = rmat12.to_c()
    a = _lib.dsp_args()
    a.matrix = ctypes.pointer(c)
    a.dims, a.task_dist, a.comm_type, a.n_rolls, a.repeat, a.n_streams = dims, 2, 2, 4, 7, 4
    a.world, a.devices, a.platform, a.b_seed, a.b_ones = world, devs, 0, 21, 0
    a.c_out = C.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    rep = _lib.dsp_report()
    _lib.call("dsp_run", ctypes.byref(a), ctypes.byref(rep))
    _check(rmat12, C, dims)
    assert rep.reps_counted == 2 and rep.avg_ms > 0 and rep.gflops > 0
    # traffic = the reference formula summed over ranks
    g_plan_traffic = 0
    from distspmm_b200.dist import build_local_group
    g = build_local_group(rmat12, world, _devices(world), dims, 4, 2, 2)
    assert rep.traffic_intra == g.traffic_intra
    assert list(rep.remap[:rep.T]) == g.plan.remap.tolist()
    g.close()


_DSP_RUN_SNIPPET = r"""
import ctypes, sys
import numpy as np
import distspmm_b200 as d, oracle
from distspmm_b200 import _lib
A = d.gen_rmat(12, seed=8)
world, dims = 4, 128
import torch
n = torch.cuda.device_count()
devs = (ctypes.c_int * world)(*[p % n for p in range(world)])
C = np.zeros((A.num_rows, dims), np.float32)
c = A.to_c()
a = _lib.dsp_args()
a.matrix = ctypes.pointer(c)
a.dims, a.task_dist, a.comm_type, a.n_rolls, a.repeat, a.n_streams = dims, 2, 2, 4, 7, 4
a.world, a.devices, a.platform, a.b_seed, a.b_ones = world, devs, 0, 21, 0
a.c_out = C.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
rep = _lib.dsp_report()
_lib.call("dsp_run", ctypes.byref(a), ctypes.byref(rep))
ref, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, d.dense_b(A.num_cols, dims, 21))
ok, worst = oracle.check_close(C, ref, ab, 1e-5)
print(int(ok and np.isfinite(C).all()), rep.traffic_intra, rep.fetched_bytes)
"""


def test_dsp_run_partition_and_fetch_scope_env(gpu):
    """The CLI pipeline's opt-in extensions (DSP_PARTITION=balanced, DSP_FETCH_SCOPE=rank,
    DSP_PIPELINE=split):
    same C as the oracle, and no more fetched bytes than the reference-semantics run."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

    def run(**env):
        e = dict(os.environ, PYTHONPATH=root, **env)
        out = subprocess.run([os.environ.get("PYTHON", "python"), "-c", _DSP_RUN_SNIPPET], env=e, cwd=root,
                             capture_output=True, text=True, timeout=600)
        assert out.returncode == 0, out.stderr[-2000:]
        ok, traffic, fetched = (int(x) for x in out.stdout.split()[-3:])
        assert ok == 1
        return traffic, fetched

    _, f_ref = run()
    _, f_rank = run(DSP_FETCH_SCOPE="rank")
    assert f_rank <= f_ref
    run(DSP_PARTITION="balanced", DSP_FETCH_SCOPE="rank")
    run(DSP_PARTITION="balanced", DSP_FETCH_SCOPE="rank", DSP_PIPELINE="split")


def test_cli_report_format(gpu, tmp_path):
    from distspmm_b200 import build
    A = d.gen_rmat(11, seed=1)
    prefix = str(tmp_path / "g")
    d.save_csr(prefix, A)
    exe = os.path.join(build.BIN, "dist_spmm_node")
    out = subprocess.run([exe, "-np", "2", prefix, "64", "2", "2", "2", "7", "4"], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.strip().splitlines()
    assert lines[0] == "task_distribution: 2 and rolls:2"
    assert len(lines[1].split()) == 4
    assert lines[2] == f"Running dist_spmm_programs on {prefix} with [64] dims".replace("_programs", " programs")
    keys = ["Processing time: (ms)", "Re-allocation time(all):", "Max memory used:", "Average time used:",
            "Communication Traffic Intra :", "Communication Traffic Inter :", "Throughput:"]
    for k, ln in zip(keys, lines[3:]):
        assert ln.startswith(k), (k, ln)
    # usage error and .mtx refusal as in the reference
    assert subprocess.run([exe, prefix], capture_output=True).returncode != 0
    assert subprocess.run([exe, "x.mtx", "64", "2", "2", "2", "7"], capture_output=True).returncode != 0


def test_bounded_wait_gives_up_with_a_status(gpu):
    """Failure detection without a fault: a fetch-style wait on an mbarrier that nothing
    completes gives up after its budget, records an error code the host reads, and leaves
    the context usable."""
    import ctypes

    import torch
    from distspmm_b200 import _lib
    code = ctypes.c_int(0)
    rc = _lib.lib().dsp_selftest_bounded_wait(2_000_000, ctypes.byref(code))  # ~1 ms budget
    assert rc == -7 and code.value == 3
    assert b"gave up" in _lib.lib().dsp_last_error()
    assert (torch.ones(4, device="cuda") * 2).sum().item() == 8
