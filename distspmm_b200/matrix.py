"""Host CSR matrices: the binary CSR format of the reference and the synthetic inputs.

``Csr`` mirrors ``SparseMatrix<int64_t, float>`` (src/sparse_matrix.h:19-65): int64
indptr / indices and fp32 values in host memory (numpy). All parsing, validation and
generation runs in the native library.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import P, c_f32, c_i64, call, dsp_csr, lib


@dataclass
class Csr:
    indptr: np.ndarray   # int64 [num_rows + 1]
    indices: np.ndarray  # int64 [nnz]
    values: np.ndarray   # float32 [nnz]
    num_rows: int
    num_cols: int

    @property
    def nnz(self) -> int:
        return int(self.indptr[-1]) if self.indptr.size else 0

    def to_c(self) -> dsp_csr:
        """A dsp_csr view of this matrix (no copy; keep self alive while it is used)."""
        self.indptr = np.ascontiguousarray(self.indptr, np.int64)
        self.indices = np.ascontiguousarray(self.indices, np.int64)
        self.values = np.ascontiguousarray(self.values, np.float32)
        if self.indices.size == 0:  # keep valid pointers for empty matrices
            self.indices = np.zeros(1, np.int64)[:0]
            self.values = np.zeros(1, np.float32)[:0]
        c = dsp_csr()
        c.num_rows = self.num_rows
        c.num_cols = self.num_cols
        c.nnz = self.nnz
        c.indptr = self.indptr.ctypes.data_as(P(c_i64))
        c.indices = self.indices.ctypes.data_as(P(c_i64))
        c.values = self.values.ctypes.data_as(P(c_f32))
        return c

    @staticmethod
    def from_c(c: dsp_csr) -> "Csr":
        """Copy a library-allocated dsp_csr into numpy arrays and free it."""
        try:
            m, z = int(c.num_rows), int(c.nnz)
            ip = np.ctypeslib.as_array(c.indptr, shape=(m + 1,)).copy()
            ix = np.ctypeslib.as_array(c.indices, shape=(max(z, 1),))[:z].copy()
            vv = np.ctypeslib.as_array(c.values, shape=(max(z, 1),))[:z].copy()
            return Csr(ip, ix, vv, m, int(c.num_cols))
        finally:
            lib().dsp_csr_free(ctypes.byref(c))

    def validate(self) -> None:
        c = self.to_c()
        call("dsp_csr_validate", ctypes.byref(c))

    def row_lengths(self) -> np.ndarray:
        return np.diff(self.indptr)


def load_from_csr(prefix: str) -> Csr:
    """SparseMatrix::load_from_csr (src/sparse_matrix.h:83-159), with validation."""
    c = dsp_csr()
    call("dsp_csr_load", str(prefix).encode(), ctypes.byref(c))
    return Csr.from_c(c)


def load_rows(prefix: str, row_lb: int, row_ub: int) -> Csr:
    """Rows [row_lb, row_ub) only (load_from_csr + turn_local_l_u_csr without reading the
    whole matrix)."""
    c = dsp_csr()
    call("dsp_csr_load_rows", str(prefix).encode(), row_lb, row_ub, ctypes.byref(c))
    return Csr.from_c(c)


def save_csr(prefix: str, a: Csr) -> None:
    c = a.to_c()
    call("dsp_csr_save", str(prefix).encode(), ctypes.byref(c))


def gen_rmat(scale: int, edge_factor: int = 16, a: float = 0.57, b: float = 0.19, c: float = 0.19,
             seed: int = 1) -> Csr:
    """Symmetrised, deduplicated R-MAT without self-loops; values U(0,1)."""
    out = dsp_csr()
    call("dsp_gen_rmat", scale, edge_factor, a, b, c, seed, ctypes.byref(out))
    return Csr.from_c(out)


def gen_stencil27(n: int, seed: int = 1) -> Csr:
    """27-point stencil on an n^3 grid: diagonal 26, off-diagonals U(-1,0)."""
    out = dsp_csr()
    call("dsp_gen_stencil27", n, seed, ctypes.byref(out))
    return Csr.from_c(out)


def gen_uniform(rows: int, nnz_per_row: int, seed: int = 1) -> Csr:
    """rows x rows with nnz_per_row distinct uniform columns per row; values U(0,1)."""
    out = dsp_csr()
    call("dsp_gen_uniform", rows, nnz_per_row, seed, ctypes.byref(out))
    return Csr.from_c(out)


def dense_b(rows: int, ncols: int, seed: int, row0: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    """Synthetic dense B rows [row0, row0 + rows): U(-1,1) from a counter hash (the same
    values the device fill produces)."""
    B = np.empty((rows, ncols), np.float32) if out is None else out
    assert B.dtype == np.float32 and B.flags.c_contiguous and B.shape == (rows, ncols)
    call("dsp_fill_dense_host", B.ctypes.data_as(P(c_f32)), row0, rows, ncols, ncols, seed)
    return B


def dense_b_rows(rows: np.ndarray, ncols: int, seed: int) -> np.ndarray:
    """The listed global rows of the synthetic dense B (the values dense_b gives them)."""
    rows = np.ascontiguousarray(rows, np.int64)
    B = np.empty((rows.size, ncols), np.float32)
    call("dsp_fill_dense_rows_host", B.ctypes.data_as(P(c_f32)), rows.ctypes.data_as(P(c_i64)), rows.size, ncols,
         ncols, seed)
    return B


def make_matrix(kind: str, seed: int = 1, **kw) -> Csr:
    """Named synthetic matrices of the benchmark configurations."""
    if kind == "rmat":
        return gen_rmat(kw.get("scale", 15), kw.get("edge_factor", 16), seed=seed)
    if kind == "stencil27":
        return gen_stencil27(kw.get("n", 32), seed=seed)
    if kind == "uniform":
        return gen_uniform(kw.get("rows", 1 << 16), kw.get("nnz_per_row", 32), seed=seed)
    raise ValueError(f"unknown matrix kind {kind!r}")
