"""The native planner is bit-exact with the oracle (and through it, with the reference's
golden vectors): tiling, needed sets, HSDMA, node merge, selector, traffic."""
import json
import os

import numpy as np
import pytest

import distspmm_b200 as d
import oracle
from distspmm_b200 import planner
from conftest import GOLDEN


@pytest.fixture(scope="module")
def rmat():
    return d.gen_rmat(13, seed=11)


def test_hsdma_matches_reference_golden():
    for c in json.load(open(os.path.join(GOLDEN, "hsdma_cases.json"))):
        got = planner.hsdma(np.array(c["demand"]), np.array(c["node_of_gpu"]), c["tasks_per_gpu"], c["max_inter"],
                            c["max_intra"])
        assert got.tolist() == c["remap"]


def test_hsdma_random_matches_oracle():
    rng = np.random.default_rng(1)
    for _ in range(200):
        P = int(rng.choice([1, 2, 4, 8]))
        rolls = int(rng.integers(1, 6))
        nodes = int(rng.choice([n for n in (1, 2, 4) if P % n == 0]))
        D = rng.integers(0, int(rng.choice([2, 100, 100000])), size=(P, P * rolls))
        node = np.repeat(np.arange(nodes), P // nodes)
        assert (planner.hsdma(D, node, rolls) == oracle.hsdma(D, node, rolls)).all()


@pytest.mark.parametrize("P,rolls", [(1, 1), (1, 4), (2, 4), (3, 2), (8, 4), (8, 1)])
def test_tiling_matches_oracle(rmat, P, rolls):
    T = P * rolls
    for r in range(P):
        lb, ub = planner.partition_bounds(rmat.num_rows, P, r)
        loc = planner.partition(rmat, lb, ub)
        a = planner.tile(loc, T)
        b = oracle.tile(loc.indptr, loc.indices, rmat.num_cols, T)
        assert a.cpt == b["cpt"]
        for k in ("n_col", "n_slice", "nnz", "offsets", "needed"):
            assert np.array_equal(getattr(a, k), b[k]), k


def test_tiling_odd_sizes():
    # columns not divisible by T, T > columns, empty local matrix
    A = d.gen_uniform(37, 5, seed=2)
    for T in (1, 4, 7, 36, 37, 50):
        a = planner.tile(A, T)
        b = oracle.tile(A.indptr, A.indices, A.num_cols, T)
        assert a.cpt == b["cpt"] and np.array_equal(a.n_col, b["n_col"]) and np.array_equal(a.needed, b["needed"])
        assert np.array_equal(a.n_slice, b["n_slice"])
    E = planner.partition(A, 5, 5)
    a = planner.tile(E, 4)
    assert a.n_col.tolist() == [0] * 4 and a.n_slice.tolist() == [0] * 4


def test_merge_matches_oracle(rmat):
    P, rolls = 4, 3
    T = P * rolls
    tl = []
    for r in range(P):
        lb, ub = planner.partition_bounds(rmat.num_rows, P, r)
        tl.append(planner.tile(planner.partition(rmat, lb, ub), T))
    counts = np.stack([t.n_col for t in tl])
    cols = np.concatenate([t.needed for t in tl])
    n1, off1, m1 = planner.merge_needed(counts, cols)
    n2, off2, m2 = oracle.merge(counts, cols, tl[0].cpt)
    assert np.array_equal(n1, n2) and np.array_equal(off1, off2) and np.array_equal(m1, m2)
    # on one node the union over all ranks is the set of nonempty columns of the whole matrix
    whole = planner.tile(rmat, T)
    assert np.array_equal(n1, whole.n_col) and np.array_equal(m1, whole.needed)


def test_selector_matches_oracle_and_golden():
    rng = np.random.default_rng(3)
    T = 64
    for platform, model in (("h100", oracle.H100_INTRA), ("a800", oracle.A800_INTRA)):
        for dims in (1, 4, 16, 32, 64, 100, 128, 256, 512):
            n_slice = rng.integers(0, 5000, T).astype(np.int32)
            n_col = (rng.random(T) * (n_slice + 1)).astype(np.int32)
            for ct in (0, 1, 2):
                a = planner.comm_select(ct, dims, n_col, n_slice, platform)
                b = oracle.select(ct, dims, model, n_col, n_slice)
                assert np.array_equal(a, b), (platform, dims, ct)
    # inter-tier decisions too
    si, se = planner.comm_select(2, 128, np.array([1, 50]), np.array([100, 60]), "h100", with_inter=True)
    assert se.tolist() == oracle.select(2, 128, oracle.H100_INTER, np.array([1, 50]), np.array([100, 60])).tolist()


def test_model_presets_are_reference_constants():
    m = planner.comm_model_preset("h100", 0)
    assert (m.a, m.b, m.c, m.u) == tuple(float(np.float32(x)) for x in oracle.H100_INTRA)
    m = planner.comm_model_preset("a800", 1)
    assert (m.a, m.b, m.c, m.u) == tuple(float(np.float32(x)) for x in oracle.A800_INTER)


def test_traffic_matches_oracle():
    rng = np.random.default_rng(4)
    for _ in range(50):
        T = 32
        remap = rng.integers(0, 8, T)
        sp = rng.integers(0, 2, T)
        n_col = rng.integers(0, 10000, T)
        n_slice = rng.integers(0, 10000, T)
        for me in range(8):
            assert planner.traffic_intra(me, remap, sp, n_col, n_slice, 128) == \
                oracle.traffic_intra(me, remap, sp, n_col, n_slice, 128)


def test_traffic_inter_formula():
    # 2 nodes x 2 ranks; rank 0's inter traffic: tiles owned by rank 2 (same position, other node)
    remap = np.array([0, 1, 2, 3, 2])
    sp = np.array([0, 0, 1, 0, 0])
    n_col = np.array([1, 1, 10, 1, 3])
    n_slice = np.array([5, 5, 50, 5, 7])
    assert planner.traffic_inter(0, 2, 2, remap, sp, n_col, n_slice, 4) == 4 * 4 * (10 + 7)
    assert planner.traffic_inter(0, 2, 1, remap, sp, n_col, n_slice, 4) == 0


def test_gflops_formula():
    assert planner.gflops(1_000_000, 128, 2.0) == pytest.approx(2.0 * 1e6 * 128 / 2.0 / 1e6)


def test_alloc_slice_and_random():
    assert planner.alloc_slice(4, 3).tolist() == [0, 0, 0, 1, 1, 1, 2, 2, 2, 3, 3, 3]
    r = planner.alloc_random(8, 4, seed=9)
    assert sorted(r.tolist()) == sorted(planner.alloc_slice(8, 4).tolist())
    assert (r == planner.alloc_random(8, 4, seed=9)).all()


@pytest.mark.parametrize("P", [1, 2, 3, 8, 64])
def test_balanced_partition_tiles_rows_with_equal_cost(rmat, P):
    """Work-balanced bounds: contiguous, in rank order, covering [0, M); every range's cost
    (nonzeros + rows) within one row of total / P."""
    ip = rmat.indptr
    M = rmat.num_rows
    b = [planner.partition_bounds_balanced(ip, P, p) for p in range(P)]
    assert b[0][0] == 0 and b[-1][1] == M
    assert all(b[p][1] == b[p + 1][0] for p in range(P - 1))
    assert all(lb <= ub for lb, ub in b)
    cost = np.asarray(ip, np.int64) + np.arange(M + 1)
    total = int(cost[-1])
    worst_row = int(np.diff(cost).max())
    for lb, ub in b:
        assert int(cost[ub] - cost[lb]) <= -(-total // P) + worst_row
    # the rule itself: rank p starts at the first row whose prefix cost reaches ceil(p * total / P)
    for p in range(1, P):
        target = -(-(total * p) // P)
        assert b[p][0] == int(np.searchsorted(cost, target, side="left"))


def test_balanced_partition_edge_cases():
    ip = np.array([0], np.int64)  # no rows
    assert planner.partition_bounds_balanced(ip, 4, 3) == (0, 0)
    ip = np.array([0, 0, 0, 5, 5], np.int64)  # empty rows and one heavy row; more ranks than rows
    b = [planner.partition_bounds_balanced(ip, 6, p) for p in range(6)]
    assert b[0][0] == 0 and b[-1][1] == 4 and all(b[p][1] == b[p + 1][0] for p in range(5))
    with pytest.raises(d.DspError):
        planner.partition_bounds_balanced(ip, 0, 0)


def test_fetch_view_scopes(rmat):
    from distspmm_b200.dist import fetch_view, global_plan
    P, rolls = 4, 2
    bounds = [planner.partition_bounds(rmat.num_rows, P, p) for p in range(P)]
    tilings = [planner.tile(planner.partition(rmat, lb, ub), P * rolls) for lb, ub in bounds]
    plan = global_plan(tilings, 2, rolls)
    assert fetch_view(plan, tilings[1], "node") is plan
    v = fetch_view(plan, tilings[1], "rank")
    assert np.array_equal(v.n_col, tilings[1].n_col) and np.array_equal(v.merged, tilings[1].needed)
    assert np.array_equal(v.remap, plan.remap) and v.T == plan.T
    # each rank's own list is a subset of the node union, tile by tile
    for t in range(plan.T):
        own = set(v.merged[v.offsets[t]:v.offsets[t + 1]].tolist())
        union = set(plan.merged[plan.offsets[t]:plan.offsets[t + 1]].tolist())
        assert own <= union
    with pytest.raises(ValueError):
        fetch_view(plan, tilings[1], "cluster")


def test_merge_matches_reference_merge_golden():
    """Node union of the ranks' needed sets: the engine's dsp_merge_needed and the oracle
    restatement against the reference's own double_level_comm_node_processing
    (src/utils.h:439-547), run with one thread per rank (tests/golden/merge_cases.json)."""
    for c in json.load(open(os.path.join(GOLDEN, "merge_cases.json"))):
        counts = np.array(c["counts"], np.int32)
        flat = np.array(c["lists"], np.int32)
        n, off, merged = planner.merge_needed(counts, flat)
        assert n.tolist() == c["merged_count"], (c["matrix"], c["P"])
        assert off.tolist() == c["offsets"] and merged.tolist() == c["merged"]
        n2, off2, m2 = oracle.merge(counts, flat, c["cpt"])
        assert n2.tolist() == c["merged_count"] and m2.tolist() == c["merged"]


def test_hsdma_mpi_wrapper_matches_reference_golden():
    """The distributed allocation (every rank computes HSDMA from the all-gathered demand)
    gives the remap that every rank holds after the reference's ComputeAllocation_HSDMA_MPI
    (Gather to the root, HSDMA there, Bcast; src/utils.h:358-437)."""
    for c in json.load(open(os.path.join(GOLDEN, "hsdma_mpi_cases.json"))):
        D = np.array(c["demand"], np.int32)
        got = planner.hierarchical_iterative_refinement_allocation(D, np.array(c["node_of_gpu"], np.int32),
                                                                   c["tasks_per_gpu"])
        assert got.tolist() == c["remap"]


@pytest.mark.skipif(oracle.ref_mpi_lib() is None, reason="reference MPI shim not built here")
def test_merge_random_vs_reference_build(rmat):
    """Live check against the reference's merge on tilings of a fresh matrix."""
    for P, rolls in ((2, 3), (5, 2)):
        T = P * rolls
        tilings = [planner.tile(planner.partition(rmat, *planner.bounds(rmat, P, p, "rows")), T) for p in range(P)]
        counts = np.stack([t.n_col for t in tilings])
        flat = np.concatenate([t.needed for t in tilings])
        want = oracle.ref_node_merge(counts, flat)
        got = planner.merge_needed(counts, flat)
        assert all(np.array_equal(a, b) for a, b in zip(got, want))
