"""CPU oracle for the distributed SpMM hot path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and the
``--impl reference`` arm) may import this package, and only as the checker or the timed
CPU baseline. The product (``distspmm_b200``) never imports it.

What it holds
  * ``liboracle.so`` (oracle.c): plain-C restatement of the reference's algorithms —
    SpMM with double accumulation (plus |A|.|B| for the tolerance), the fp32 OpenMP CPU
    baseline, tiling / needed sets, HSDMA, node merge, the adaptive selector and the
    traffic formula — each function citing the reference file:line it follows.
  * ``libdsp_ref.so`` (ref_shim.cpp, optional): the reference's own ``src/h_sdma.h`` and
    ``src/sparse_matrix.h`` compiled from the reference sources, used to pin the
    restatement (HSDMA, loader) and to generate the golden fixtures.
  * ``libdsp_ref_mpi.so`` (ref_mpi_shim.cu, optional): the reference's MPI-bound
    ``src/utils.h`` (node merge, HSDMA MPI wrapper) compiled against the thread-rank MPI
    stand-in of ``mpi_stub/`` and run with one thread per rank.

Parity: HSDMA, its MPI wrapper, the node merge and the loader are pinned to the reference
build; tiling (inside the reference's main()), selector and traffic restate code that
cannot be built here; SpMM values are
"parity unpinned" against the reference (it never checks C) and use the elementwise
bound max|dC| <= 1e-5 * (|A|.|B|).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = os.path.join(_HERE, "_build", "liboracle.so")
_REF = os.path.join(_HERE, "_ref", "libdsp_ref.so")
_REF_MPI = os.path.join(_HERE, "_ref", "libdsp_ref_mpi.so")

_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)

_lib = None
_ref = None
_ref_mpi = None


def build(ref: bool = True, ref_src: str | None = None) -> None:
    """Compile liboracle.so (and the reference shim when the reference tree exists; its
    src/ directory is ``ref_src`` or the DSP_REFERENCE_SRC environment variable)."""
    subprocess.run(["make", "-s", "-C", _HERE, "oracle"], check=True)
    src = ref_src or os.environ.get("DSP_REFERENCE_SRC")
    if ref and src:
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF_SRC={src}"], check=True)


def _p(a, t):
    return a.ctypes.data_as(t)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB):
            build(ref=False)
        L = ctypes.CDLL(_LIB)
        L.orc_spmm_f64.argtypes = [ctypes.c_int64, _i64p, _i64p, _f32p, _f32p, ctypes.c_int64,
                                   ctypes.c_int64, _f64p, _f64p]
        L.orc_spmm_f32.argtypes = [ctypes.c_int64, _i64p, _i64p, _f32p, _f32p, ctypes.c_int64,
                                   ctypes.c_int64, _f32p, ctypes.c_int]
        L.orc_max_threads.restype = ctypes.c_int
        L.orc_partition_bounds.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int, _i64p, _i64p]
        L.orc_cpt.restype = ctypes.c_int64
        L.orc_cpt.argtypes = [ctypes.c_int64, ctypes.c_int]
        L.orc_tile.argtypes = [ctypes.c_int64, _i64p, _i64p, ctypes.c_int64, ctypes.c_int, _i32p,
                               _i32p, _i64p, _i64p, _i32p]
        L.orc_hsdma.argtypes = [_i32p, ctypes.c_int, ctypes.c_int, _i32p, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, _i32p]
        L.orc_merge.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int64, _i32p, _i32p, _i32p,
                                _i64p, _i32p]
        L.orc_threshold.restype = ctypes.c_float
        L.orc_threshold.argtypes = [ctypes.c_float] * 4 + [ctypes.c_int]
        L.orc_select.argtypes = [ctypes.c_int, ctypes.c_int] + [ctypes.c_float] * 4 + [
            ctypes.c_int, _i32p, _i32p, _u8p]
        L.orc_traffic_intra.restype = ctypes.c_int64
        L.orc_traffic_intra.argtypes = [ctypes.c_int, ctypes.c_int, _i32p, _u8p, _i32p, _i32p,
                                        ctypes.c_int]
        _lib = L
    return _lib


def ref_lib():
    """The reference's own headers behind ref_shim.cpp, or None if not built here."""
    global _ref
    if _ref is None and os.path.exists(_REF):
        R = ctypes.CDLL(_REF)
        R.ref_hsdma.argtypes = [_i32p, ctypes.c_int, ctypes.c_int, _i32p, ctypes.c_int,
                                ctypes.c_int, ctypes.c_int, _i32p]
        R.ref_load_csr.argtypes = [ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64, _i64p, _i64p,
                                   _i64p, _i64p, _i64p, _f32p]
        _ref = R
    return _ref


def ref_mpi_lib():
    """The reference's MPI-bound utils.h behind ref_mpi_shim.cu, or None if not built here."""
    global _ref_mpi
    if _ref_mpi is None and os.path.exists(_REF_MPI):
        R = ctypes.CDLL(_REF_MPI)
        R.ref_node_merge.argtypes = [ctypes.c_int, ctypes.c_int, _i32p, _i32p, _i32p, _i64p, _i32p]
        R.ref_hsdma_mpi.argtypes = [ctypes.c_int, ctypes.c_int, _i32p, _i32p, ctypes.c_int, _i32p]
        _ref_mpi = R
    return _ref_mpi


def ref_node_merge(counts, cols):
    """double_level_comm_node_processing (src/utils.h:439-547) of the reference, on one
    thread per rank. counts: R x T pre-merge sizes; cols: flat rank-major, tile-major lists.
    Returns (merged counts, offsets, merged lists ascending) like merge()."""
    R = ref_mpi_lib()
    if R is None:
        raise RuntimeError("reference MPI shim not built")
    counts = np.ascontiguousarray(counts, np.int32)
    cols = np.ascontiguousarray(cols, np.int32) if np.size(cols) else np.zeros(1, np.int32)
    P, T = counts.shape
    n = np.zeros(T, np.int32)
    off = np.zeros(T + 1, np.int64)
    if R.ref_node_merge(P, T, _p(counts, _i32p), _p(cols, _i32p), _p(n, _i32p), _p(off, _i64p), None) != 0:
        raise RuntimeError("ranks disagree after the reference merge")
    out = np.zeros(max(int(off[-1]), 1), np.int32)
    R.ref_node_merge(P, T, _p(counts, _i32p), _p(cols, _i32p), _p(n, _i32p), _p(off, _i64p), _p(out, _i32p))
    return n, off, out[: int(off[-1])]


def ref_hsdma_mpi(demand, node_of_gpu, tasks_per_gpu):
    """ComputeAllocation_HSDMA_MPI (src/utils.h:358-437) of the reference, on one thread per
    rank, each with its own demand row. Returns the P x T remap every rank holds."""
    R = ref_mpi_lib()
    if R is None:
        raise RuntimeError("reference MPI shim not built")
    demand = np.ascontiguousarray(demand, np.int32)
    P, T = demand.shape
    nodes = np.ascontiguousarray(node_of_gpu, np.int32)
    remap = np.zeros(P * T, np.int32)
    R.ref_hsdma_mpi(P, T, _p(demand, _i32p), _p(nodes, _i32p), tasks_per_gpu, _p(remap, _i32p))
    return remap.reshape(P, T)


# ---------------------------------------------------------------- SpMM

def spmm_f64(indptr, indices, values, B, N=None):
    """Return (C, Cabs) in float64: C = A.B and Cabs = |A|.|B| (for the tolerance)."""
    indptr = np.ascontiguousarray(indptr, np.int64)
    indices = np.ascontiguousarray(indices, np.int64)
    values = np.ascontiguousarray(values, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    m = indptr.shape[0] - 1
    N = B.shape[1] if N is None else N
    C = np.empty((m, N), np.float64)
    Ca = np.empty((m, N), np.float64)
    lib().orc_spmm_f64(m, _p(indptr, _i64p), _p(indices, _i64p), _p(values, _f32p), _p(B, _f32p),
                       B.shape[1], N, _p(C, _f64p), _p(Ca, _f64p))
    return C, Ca


def spmm_f32(indptr, indices, values, B, threads: int = 0, out=None):
    """fp32 OpenMP CSR x dense loop — the timed CPU baseline."""
    m = indptr.shape[0] - 1
    N = B.shape[1]
    C = np.empty((m, N), np.float32) if out is None else out
    lib().orc_spmm_f32(m, _p(indptr, _i64p), _p(indices, _i64p), _p(values, _f32p), _p(B, _f32p),
                       B.shape[1], N, _p(C, _f32p), threads)
    return C


def max_threads() -> int:
    return int(lib().orc_max_threads())


def check_close(C_dev, C_ref, C_abs, rel: float = 1e-5):
    """Elementwise bound |C_dev - C_ref| <= rel * (|A|.|B|) (+ tiny absolute slack for
    rows whose bound is exactly 0). Returns (ok, worst_ratio)."""
    diff = np.abs(C_dev.astype(np.float64) - C_ref)
    bound = rel * C_abs + 1e-30
    ratio = diff / bound
    worst = float(ratio.max()) if ratio.size else 0.0
    return worst <= 1.0, worst


def sample_rows(num_rows, frac=0.01, indptr=None, min_degree=None, offset=0):
    """Rows to check at sizes where a full CPU product is too slow: every k-th row
    (k = 1/frac, starting at `offset`), plus every row holding more than `min_degree`
    nonzeros when indptr is given (the hub rows of power-law matrices)."""
    k = max(1, int(round(1.0 / frac)))
    rows = np.arange(offset % k, num_rows, k, dtype=np.int64)
    if indptr is not None and min_degree is not None:
        heavy = np.nonzero(np.diff(np.asarray(indptr, np.int64)) > min_degree)[0]
        rows = np.union1d(rows, heavy)
    return rows


def check_rows(indptr, indices, values, B, rows, C_rows, rel: float = 1e-5):
    """check_close of C_rows (the device result at `rows` of a CSR) against the oracle
    computed on those rows only. B is the dense operand, or a function returning the B
    rows of a list of column ids (so that B never has to exist whole on the host).
    Returns (ok, worst_ratio)."""
    indptr = np.asarray(indptr, np.int64)
    rows = np.asarray(rows, np.int64)
    lens = indptr[rows + 1] - indptr[rows]
    ip = np.zeros(rows.size + 1, np.int64)
    np.cumsum(lens, out=ip[1:])
    if rows.size and ip[-1] > 0:
        starts = np.repeat(indptr[rows] - ip[:-1], lens)
        sel = np.arange(ip[-1], dtype=np.int64) + starts
    else:
        sel = np.zeros(0, np.int64)
    cols = np.asarray(indices)[sel]
    if callable(B):
        uniq, cols = np.unique(cols, return_inverse=True)
        B = B(uniq) if uniq.size else np.zeros((1, np.asarray(C_rows).shape[1]), np.float32)
    ref, ab = spmm_f64(ip, cols, np.asarray(values)[sel], B)
    return check_close(np.asarray(C_rows), ref, ab, rel)


# ---------------------------------------------------------------- planning

def partition_bounds(M, P, rank):
    lb = ctypes.c_int64()
    ub = ctypes.c_int64()
    lib().orc_partition_bounds(M, P, rank, ctypes.byref(lb), ctypes.byref(ub))
    return lb.value, ub.value


def tile(indptr, indices, ncols, T):
    """Return dict(cpt, n_col, n_slice, nnz, offsets, needed) per the reference tiling."""
    indptr = np.ascontiguousarray(indptr, np.int64)
    indices = np.ascontiguousarray(indices, np.int64)
    m = indptr.shape[0] - 1
    cpt = int(lib().orc_cpt(ncols, T))
    n_col = np.zeros(T, np.int32)
    n_slice = np.zeros(T, np.int32)
    nnz = np.zeros(T, np.int64)
    lib().orc_tile(m, _p(indptr, _i64p), _p(indices, _i64p), ncols, T, _p(n_col, _i32p),
                   _p(n_slice, _i32p), _p(nnz, _i64p), None, None)
    offsets = np.zeros(T + 1, np.int64)
    needed = np.zeros(max(int(n_col.sum()), 1), np.int32)
    lib().orc_tile(m, _p(indptr, _i64p), _p(indices, _i64p), ncols, T, _p(n_col, _i32p),
                   _p(n_slice, _i32p), _p(nnz, _i64p), _p(offsets, _i64p), _p(needed, _i32p))
    return dict(cpt=cpt, n_col=n_col, n_slice=n_slice, nnz=nnz, offsets=offsets,
                needed=needed[: int(offsets[-1])])


def hsdma(demand, node_of_gpu, tasks_per_gpu, max_inter=5, max_intra=5, use_ref=False):
    demand = np.ascontiguousarray(demand, np.int32)
    P, T = demand.shape
    nodes = np.ascontiguousarray(node_of_gpu, np.int32)
    remap = np.zeros(T, np.int32)
    L = ref_lib() if use_ref else lib()
    if L is None:
        raise RuntimeError("reference shim not built")
    fn = L.ref_hsdma if use_ref else L.orc_hsdma
    fn(_p(demand, _i32p), P, T, _p(nodes, _i32p), tasks_per_gpu, max_inter, max_intra,
       _p(remap, _i32p))
    return remap


def merge(counts, cols, cpt):
    """counts: R x T; cols: flat rank-major lists. Returns (n_col_merged, offsets, merged)."""
    counts = np.ascontiguousarray(counts, np.int32)
    cols = np.ascontiguousarray(cols, np.int32)
    if cols.size == 0:
        cols = np.zeros(1, np.int32)
    R, T = counts.shape
    n = np.zeros(T, np.int32)
    off = np.zeros(T + 1, np.int64)
    lib().orc_merge(R, T, cpt, _p(counts, _i32p), _p(cols, _i32p), _p(n, _i32p), _p(off, _i64p),
                    None)
    merged = np.zeros(max(int(off[-1]), 1), np.int32)
    lib().orc_merge(R, T, cpt, _p(counts, _i32p), _p(cols, _i32p), _p(n, _i32p), _p(off, _i64p),
                    _p(merged, _i32p))
    return n, off, merged[: int(off[-1])]


def threshold(model, dims):
    a, b, c, u = model
    return float(lib().orc_threshold(a, b, c, u, dims))


def select(comm_type, dims, model, n_col, n_slice):
    n_col = np.ascontiguousarray(n_col, np.int32)
    n_slice = np.ascontiguousarray(n_slice, np.int32)
    out = np.zeros(n_col.shape[0], np.uint8)
    a, b, c, u = model
    rc = lib().orc_select(comm_type, dims, a, b, c, u, n_col.shape[0], _p(n_col, _i32p),
                          _p(n_slice, _i32p), _p(out, _u8p))
    if rc != 0:
        raise ValueError("bad comm_type")
    return out


def traffic_intra(me, remap, sparse, n_col, n_slice, dims):
    remap = np.ascontiguousarray(remap, np.int32)
    sparse = np.ascontiguousarray(sparse, np.uint8)
    n_col = np.ascontiguousarray(n_col, np.int32)
    n_slice = np.ascontiguousarray(n_slice, np.int32)
    return int(lib().orc_traffic_intra(me, remap.shape[0], _p(remap, _i32p), _p(sparse, _u8p),
                                       _p(n_col, _i32p), _p(n_slice, _i32p), dims))


def ref_load(prefix, lb=-1, ub=-1):
    """Load through the reference's own SparseMatrix::load_from_csr (+ turn_local)."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("reference shim not built")
    m = ctypes.c_int64()
    n = ctypes.c_int64()
    z = ctypes.c_int64()
    rc = R.ref_load_csr(prefix.encode(), lb, ub, ctypes.byref(m), ctypes.byref(n),
                        ctypes.byref(z), None, None, None)
    if rc != 0:
        return None
    ip = np.zeros(m.value + 1, np.int64)
    ix = np.zeros(max(z.value, 1), np.int64)
    vv = np.zeros(max(z.value, 1), np.float32)
    R.ref_load_csr(prefix.encode(), lb, ub, ctypes.byref(m), ctypes.byref(n), ctypes.byref(z),
                   _p(ip, _i64p), _p(ix, _i64p), _p(vv, _f32p))
    return dict(num_rows=m.value, num_cols=n.value, nnz=z.value, indptr=ip,
                indices=ix[: z.value], values=vv[: z.value])


# Model constants of the reference (src/comm_man.h:387-395). They are float variables
# initialised from these decimal literals.
H100_INTRA = (12873.61472, 125.27085, 105.50392, -4.65)
H100_INTER = (1452.17110, -1407.82558, 47.34021, -1.00)
A800_INTRA = (4075.35, 119.61, 98.21, -3.78)
A800_INTER = (1440.80, -1394.99, 43.65, -1.00)
