"""Synthetic inputs: structure and determinism (host-side)."""
import numpy as np

import distspmm_b200 as d


def test_rmat_structure_and_determinism():
    A = d.gen_rmat(12, seed=5)
    B = d.gen_rmat(12, seed=5)
    assert np.array_equal(A.indptr, B.indptr) and np.array_equal(A.indices, B.indices)
    assert np.array_equal(A.values, B.values)
    A.validate()
    import scipy.sparse as sp
    S = sp.csr_matrix((np.ones(A.nnz), A.indices, A.indptr), shape=(A.num_rows, A.num_cols))
    assert (S != S.T).nnz == 0          # symmetrised pattern
    assert S.diagonal().sum() == 0      # no self-loops
    for r in range(0, A.num_rows, 97):  # ascending unique columns
        c = A.indices[A.indptr[r]:A.indptr[r + 1]]
        assert np.all(np.diff(c) > 0)
    assert A.values.min() >= 0 and A.values.max() < 1
    assert A.row_lengths()[0] == A.row_lengths().max()  # a = 0.57: vertex 0 is the hub
    assert not np.array_equal(d.gen_rmat(12, seed=6).indices[:100], A.indices[:100])


def test_stencil_structure():
    n = 7
    A = d.gen_stencil27(n, seed=1)
    assert A.num_rows == n ** 3 and A.nnz == (3 * n - 2) ** 3
    A.validate()
    r = (3 * n + 3) * n + 3  # interior point
    cols = A.indices[A.indptr[r]:A.indptr[r + 1]]
    vals = A.values[A.indptr[r]:A.indptr[r + 1]]
    assert len(cols) == 27 and np.all(np.diff(cols) > 0)
    assert vals[cols == r][0] == 26.0
    off = vals[cols != r]
    assert np.all(off <= 0) and np.all(off > -1)


def test_uniform_structure():
    A = d.gen_uniform(1000, 32, seed=4)
    A.validate()
    assert np.all(A.row_lengths() == 32)
    for r in range(0, 1000, 50):
        assert np.all(np.diff(A.indices[A.indptr[r]:A.indptr[r + 1]]) > 0)


def test_dense_b_values():
    B = d.dense_b(64, 33, seed=2)
    assert B.min() >= -1 and B.max() < 1
    assert np.array_equal(B[10:20], d.dense_b(10, 33, seed=2, row0=10))
    # exact multiples of 2^-23 (24-bit uniforms scaled to (-1, 1))
    assert np.all((B.astype(np.float64) * 2 ** 23) == np.round(B.astype(np.float64) * 2 ** 23))
