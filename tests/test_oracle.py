"""Pin the CPU oracle to the reference: golden vectors produced by the reference's own
h_sdma.h / sparse_matrix.h (compiled from its sources) and by an nvcc-compiled probe of
the selector expression; plus hand-checked known answers for the restated parts."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from conftest import GOLDEN


def _golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def test_oracle_hsdma_matches_reference_golden():
    cases = _golden("hsdma_cases.json")
    assert len(cases) >= 50
    for c in cases:
        got = oracle.hsdma(np.array(c["demand"]), np.array(c["node_of_gpu"]), c["tasks_per_gpu"], c["max_inter"],
                           c["max_intra"])
        assert got.tolist() == c["remap"], c


def test_oracle_threshold_matches_nvcc_probe():
    t = _golden("thresholds.json")
    for name, v in t.items():
        for dims, bits in v["thr_bits"].items():
            mine = oracle.threshold(v["model"], int(dims))
            assert "%08x" % struct.unpack("<I", struct.pack("<f", mine))[0] == bits, (name, dims)


def test_oracle_tiling_known_answer():
    # 3 rows x 8 columns, T = 3 -> cpt = ceil(8/3) = 3; tiles [0,3) [3,6) [6,8)
    indptr = np.array([0, 3, 5, 6])
    indices = np.array([0, 4, 7, 4, 5, 1])
    t = oracle.tile(indptr, indices, 8, 3)
    assert t["cpt"] == 3
    assert t["n_col"].tolist() == [2, 2, 1]          # {0,1}, {4%3,5%3}={1,2}, {7%3}={1}
    assert t["nnz"].tolist() == [2, 3, 1]
    assert t["n_slice"].tolist() == [3, 3, 2]        # last tile min(3, 8-6) = 2
    assert t["needed"].tolist() == [0, 1, 1, 2, 1]
    # a tile without local nonzeros keeps n_slice = 0 (src/dist_spmm_node.cu:210-223)
    t2 = oracle.tile(np.array([0, 1]), np.array([0]), 8, 3)
    assert t2["n_slice"].tolist() == [3, 0, 0]


def test_oracle_merge_known_answer():
    counts = np.array([[2, 1], [1, 2]])
    cols = np.array([0, 2, 1,   2, 0, 1])  # rank0: t0={0,2}, t1={1}; rank1: t0={2}, t1={0,1}
    n, off, merged = oracle.merge(counts, cols, 3)
    assert n.tolist() == [2, 2]
    assert merged.tolist() == [0, 2, 0, 1]


def test_oracle_select_and_traffic_known_answer():
    thr = oracle.threshold(oracle.H100_INTRA, 128)
    assert 0.83 < thr < 0.85  # the README's critical density at dims 128 (~0.83)
    n_col = np.array([10, 90, 0, 5])
    n_slice = np.array([99, 99, 0, 0])
    sp = oracle.select(2, 128, oracle.H100_INTRA, n_col, n_slice)
    # d = 10/100 = 0.1 < thr -> sparse; 90/100 = 0.9 > thr -> bulk; 0/1 -> sparse; 5/1 -> bulk
    assert sp.tolist() == [1, 0, 1, 0]
    assert oracle.select(0, 128, oracle.H100_INTRA, n_col, n_slice).tolist() == [0, 0, 0, 0]
    assert oracle.select(1, 128, oracle.H100_INTRA, n_col, n_slice).tolist() == [1, 1, 1, 1]
    remap = np.array([0, 1, 1, 0])
    # rank 0 pays tiles 1 (bulk: 99 rows) and 2 (sparse: 0 rows)
    assert oracle.traffic_intra(0, remap, sp, n_col, n_slice, 128) == 4 * 128 * 99


def test_oracle_spmm_known_answer():
    # [[1, 2], [0, 3]] x [[1, 1], [2, -1]]
    ip = np.array([0, 2, 3])
    ix = np.array([0, 1, 1])
    vv = np.array([1, 2, 3], np.float32)
    B = np.array([[1, 1], [2, -1]], np.float32)
    C, Ca = oracle.spmm_f64(ip, ix, vv, B)
    assert C.tolist() == [[5, -1], [6, -3]]
    assert Ca.tolist() == [[5, 3], [6, 3]]
    C32 = oracle.spmm_f32(ip, ix, vv, B, threads=2)
    assert C32.tolist() == [[5, -1], [6, -3]]


def test_oracle_loader_golden_matches_reference_json():
    """The committed CSR files, read by the reference loader, gave csr_small_ref.json."""
    ref = _golden("csr_small_ref.json")
    ip = np.fromfile(os.path.join(GOLDEN, "csr_small_indptr.bin"), np.int64)
    ix = np.fromfile(os.path.join(GOLDEN, "csr_small_indices.bin"), np.int64)
    vv = np.fromfile(os.path.join(GOLDEN, "csr_small_values.bin"), np.float32)
    w = ref["whole"]
    assert w["num_rows"] == ip.size - 1 and w["num_cols"] == ip.size - 1 and w["nnz"] == ip[-1]
    assert np.array_equal(w["indptr"], ip) and np.array_equal(w["indices"], ix)
    assert np.array_equal(np.array(w["values"], np.float32), vv)
    for p in ref["parts"]:
        assert (p["lb"], p["ub"]) == oracle.partition_bounds(w["num_rows"], 3, ref["parts"].index(p))


@pytest.mark.skipif(oracle.ref_lib() is None, reason="reference shim not built here")
def test_oracle_hsdma_random_vs_reference_build():
    rng = np.random.default_rng(5)
    for _ in range(100):
        P = int(rng.choice([2, 4, 8]))
        rolls = int(rng.integers(1, 5))
        nodes = int(rng.choice([n for n in (1, 2) if P % n == 0]))
        D = rng.integers(0, 20, size=(P, P * rolls))
        node = np.repeat(np.arange(nodes), P // nodes)
        assert (oracle.hsdma(D, node, rolls) == oracle.hsdma(D, node, rolls, use_ref=True)).all()


def test_check_rows_matches_full_product_on_the_sample():
    """The sampled-row checker used at full benchmark sizes computes the same rows as the
    full oracle product, and flags a planted error (planted in the oracle's output, on the
    CPU)."""
    import distspmm_b200 as d
    A = d.gen_rmat(11, seed=3)
    B = d.dense_b(A.num_cols, 24, seed=4)
    C, _ = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    rows = oracle.sample_rows(A.num_rows, 0.05, A.indptr, 64, offset=3)
    assert 3 in rows and 23 in rows and (np.diff(A.indptr)[rows] > 64).sum() == (np.diff(A.indptr) > 64).sum()
    ok, worst = oracle.check_rows(A.indptr, A.indices, A.values, B, rows, C[rows].astype(np.float32))
    assert ok and worst < 0.1
    bad = C[rows].astype(np.float32)
    hub = int(np.argmax(np.diff(A.indptr)[rows]))
    bad[hub, 5] += 1e-2
    ok, worst = oracle.check_rows(A.indptr, A.indices, A.values, B, rows, bad)
    assert not ok and worst > 1.0


def test_check_rows_with_b_rows_on_demand():
    """The checker can take B as a row source (global ids -> rows), as the benchmark does
    at sizes where B is not materialised on the host; the result equals the full-B check."""
    import distspmm_b200 as d
    A = d.gen_uniform(3000, 7, seed=5)
    B = d.dense_b(A.num_cols, 16, seed=9)
    C, _ = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    rows = oracle.sample_rows(A.num_rows, 0.1, offset=1)
    full = oracle.check_rows(A.indptr, A.indices, A.values, B, rows, C[rows].astype(np.float32))
    lazy = oracle.check_rows(A.indptr, A.indices, A.values, lambda r: d.dense_b_rows(r, 16, 9), rows,
                             C[rows].astype(np.float32))
    assert full[0] and lazy[0] and abs(full[1] - lazy[1]) < 1e-12
    assert np.array_equal(d.dense_b_rows(np.array([5, 0, 2999]), 16, 9), B[[5, 0, 2999]])
