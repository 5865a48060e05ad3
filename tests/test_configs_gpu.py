"""Parity at the full sizes of the benchmark configurations (through the C ABI).

Each configuration's matrix and dense B are generated at their real sizes; C is computed
by the sm_100a kernels and compared with the CPU oracle (double accumulation) within
|dC| <= 1e-5 * (|A|.|B|) elementwise:
  1  R-MAT scale 15, N = 32: every row.
  2  R-MAT scale 20, N = 128: a 1 % strided row sample plus every row of degree > 4096
     (the hub rows that nnz-split chunks cut into pieces), on one GPU and as 8 ranks with
     the reference's semantics (equal-row partition, node-merged lists, HSDMA, adaptive
     fetch; remote rows NaN-poisoned before the step).
  3  27-point stencil 160^3 (4,096,000 rows), N = 128: 1 % strided rows.
  4  uniform 4,194,304 x 4,194,304, 32 per row, N = 256: 1 % strided rows.
  5  R-MAT scale 24 (16.8 M rows, ~520 M nonzeros), N = 128: 1 % strided rows plus every
     row of degree > 16384.
"""
import numpy as np
import pytest

import distspmm_b200 as d
import oracle

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _single_gpu_check(A, N, rows, seed=5):
    import torch
    from distspmm_b200.spmm import SpmmPlan
    B = d.dense_b(A.num_cols, N, seed)
    plan = SpmmPlan(A, 0, N)
    Bt = torch.from_numpy(B).cuda()
    C = torch.full((A.num_rows, N), float("nan"), device="cuda")
    plan(Bt, C)
    got = C[torch.from_numpy(rows).cuda()].cpu().numpy()
    info = plan.info()
    plan.close()
    del Bt, C
    torch.cuda.empty_cache()
    assert np.isfinite(got).all(), "a sampled row was not written"
    ok, worst = oracle.check_rows(A.indptr, A.indices, A.values, B, rows, got, RTOL)
    assert ok, f"worst |dC| / (1e-5 |A||B|) = {worst:.3f} over {rows.size} rows"
    return info


def test_config1_rmat15_n32_every_row(gpu):
    A = d.gen_rmat(15, seed=1)
    rows = np.arange(A.num_rows)
    _single_gpu_check(A, 32, rows)


@pytest.fixture(scope="module")
def rmat20():
    return d.gen_rmat(20, seed=1)


def test_config2_rmat20_n128_sample_and_hubs(gpu, rmat20):
    A = rmat20
    rows = oracle.sample_rows(A.num_rows, 0.01, A.indptr, 4096)
    assert (np.diff(A.indptr)[rows] > 4096).sum() >= 10  # the hub rows are in the sample
    info = _single_gpu_check(A, 128, rows)
    assert info["variant"] == 1 and info["split_rows"] > 0  # nnz-split, hub rows cut into pieces


def test_config2_rmat20_eight_ranks_reference_semantics(gpu, rmat20):
    import torch
    from distspmm_b200.dist import build_local_group
    A, N, seed = rmat20, 128, 7
    g = build_local_group(A, 8, [0] * 8, N, n_rolls=4, task_dist=2, comm_type=2, partition="rows",
                          fetch_scope="node")
    for r in g.ranks:
        r.poison_remote()
        r.fill_b(seed)
    torch.cuda.synchronize()
    g.step()
    torch.cuda.synchronize()
    B = d.dense_b(A.num_cols, N, seed)
    for p, (r, (lb, ub)) in enumerate(zip(g.ranks, g.bounds)):
        r.check_error()
        part = np.empty((ub - lb, N), np.float32)
        r.download_c(part)
        torch.cuda.synchronize()
        local = np.arange(lb, ub)
        rows = local[oracle.sample_rows(ub - lb, 0.01, A.indptr[lb:ub + 1], 4096, offset=p)]
        got = part[rows - lb]
        assert np.isfinite(got).all(), f"rank {p}: a remote row was used before it was fetched"
        ok, worst = oracle.check_rows(A.indptr, A.indices, A.values, B, rows, got, RTOL)
        assert ok, f"rank {p}: worst {worst:.3f}"
    g.close()


def test_config3_stencil160_n128_sample(gpu):
    A = d.gen_stencil27(160, seed=1)
    assert A.num_rows == 4_096_000 and A.nnz == 478 ** 3
    info = _single_gpu_check(A, 128, oracle.sample_rows(A.num_rows, 0.01))
    assert info["variant"] == 0  # row-split for the banded matrix


def test_config4_uniform_n256_sample(gpu):
    A = d.gen_uniform(1 << 22, 32, seed=1)
    _single_gpu_check(A, 256, oracle.sample_rows(A.num_rows, 0.01))


def test_config5_rmat24_n128_sample_and_hubs(gpu):
    A = d.gen_rmat(24, seed=1)
    rows = oracle.sample_rows(A.num_rows, 0.01, A.indptr, 16384)
    _single_gpu_check(A, 128, rows)
