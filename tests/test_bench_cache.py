"""bench.py's --csr-cache: a generated matrix stored as the reference's binary CSR files and
read back by a later run is the same matrix (CPU only: generation and file I/O are host code)."""
import types

import numpy as np

import bench


def _args(tmp_path, **kw):
    a = dict(csr_cache=str(tmp_path), matrix="rmat", scale=10, seed=3, grid=6, rows=512, nnz_per_row=4, dims=64)
    a.update(kw)
    return types.SimpleNamespace(**a)


def test_csr_cache_round_trip(tmp_path):
    for kw in ({}, {"matrix": "stencil27"}, {"matrix": "uniform"}):
        a = _args(tmp_path, **kw)
        A1 = bench.load_local(a, 0, 1, None)[0]
        assert (tmp_path / bench.matrix_key(a) / "A_indptr.bin").exists()
        A2 = bench.load_local(a, 0, 1, None)[0]  # read back from the cache
        ref = bench.make_workload(a)
        for A in (A1, A2):
            assert A.num_rows == ref.num_rows and A.nnz == ref.nnz
            assert np.array_equal(A.indptr, ref.indptr)
            assert np.array_equal(A.indices, ref.indices)
            assert np.array_equal(A.values, ref.values)


def test_matrix_key_separates_seeds_and_shapes(tmp_path):
    keys = {bench.matrix_key(_args(tmp_path, **kw)) for kw in
            ({}, {"seed": 4}, {"scale": 11}, {"matrix": "stencil27"}, {"matrix": "stencil27", "grid": 7},
             {"matrix": "uniform"}, {"matrix": "uniform", "nnz_per_row": 5})}
    assert len(keys) == 7
