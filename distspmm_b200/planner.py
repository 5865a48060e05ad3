"""Integer planning of the distributed SpMM (host, bit-exact with the reference).

Python face of the native planner, named after the reference functions it replaces:
  partition_bounds / partition     src/dist_spmm_node.cu:85-93, src/sparse_matrix.h:178-199
  tile_counts / tile_needed        src/dist_spmm_node.cu:103-132, :210-223
  hierarchical_iterative_refinement_allocation   src/h_sdma.h:78-228
  alloc_slice / alloc_random       src/dist_spmm_node.cu:140-149
  double_level_comm_node_processing (merge)      src/utils.h:439-547
  comm_model_preset / comm_select  src/comm_man.h:369-410
  traffic_intra / traffic_inter    src/comm_man.h:508-542
  gflops                           src/dist_spmm_node.cu:435
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import PLATFORM, P, c_i32, c_i64, call, dsp_comm_model, dsp_csr, lib
from .matrix import Csr

_u8p = P(ctypes.c_uint8)


def _i32(a):
    return np.ascontiguousarray(a, np.int32)


def _ptr(a, t):
    return a.ctypes.data_as(P(t))


def partition_bounds(M: int, P_: int, rank: int):
    lb, ub = c_i64(), c_i64()
    call("dsp_partition_bounds", M, P_, rank, ctypes.byref(lb), ctypes.byref(ub))
    return lb.value, ub.value


def partition_bounds_balanced(indptr: np.ndarray, P_: int, rank: int):
    """Contiguous rows of equal cost (nonzeros + rows); not in the reference (an addition
    for skewed graphs, where the equal-row split of partition_bounds overloads rank 0)."""
    ip = np.ascontiguousarray(indptr, np.int64)
    lb, ub = c_i64(), c_i64()
    call("dsp_partition_bounds_balanced", _ptr(ip, c_i64), ip.size - 1, P_, rank, ctypes.byref(lb),
         ctypes.byref(ub))
    return lb.value, ub.value


PARTITIONS = ("rows", "balanced")


def bounds(g: Csr, P_: int, rank: int, how: str = "rows"):
    """Row range of `rank`: the reference's equal-row split ("rows") or the work-balanced
    one ("balanced")."""
    if how == "rows":
        return partition_bounds(g.num_rows, P_, rank)
    if how == "balanced":
        return partition_bounds_balanced(g.indptr, P_, rank)
    raise ValueError(f"partition {how!r}: expected one of {PARTITIONS}")


def partition(g: Csr, lb: int, ub: int) -> Csr:
    c = g.to_c()
    out = dsp_csr()
    call("dsp_partition", ctypes.byref(c), lb, ub, ctypes.byref(out))
    return Csr.from_c(out)


@dataclass
class Tiling:
    cpt: int
    n_col: np.ndarray    # int32 [T] pre-merge distinct columns per tile
    n_slice: np.ndarray  # int32 [T]
    nnz: np.ndarray      # int64 [T]
    offsets: np.ndarray  # int64 [T+1]
    needed: np.ndarray   # int32 flat, ascending tile-local ids


def tile(local: Csr, T: int) -> Tiling:
    c = local.to_c()
    cpt = c_i64()
    n_col = np.zeros(T, np.int32)
    n_slice = np.zeros(T, np.int32)
    nnz = np.zeros(T, np.int64)
    call("dsp_tile_counts", ctypes.byref(c), T, ctypes.byref(cpt), _ptr(n_col, c_i32), _ptr(n_slice, c_i32),
         _ptr(nnz, c_i64))
    off = np.zeros(T + 1, np.int64)
    call("dsp_tile_needed", ctypes.byref(c), T, _ptr(off, c_i64), None)
    needed = np.zeros(max(int(off[-1]), 1), np.int32)
    call("dsp_tile_needed", ctypes.byref(c), T, _ptr(off, c_i64), _ptr(needed, c_i32))
    return Tiling(int(cpt.value), n_col, n_slice, nnz, off, needed[: int(off[-1])])


def col_presence(d_cols, num_cols: int, stream: int = 0):
    """Device byte map of the columns in d_cols (a CUDA int64 tensor): 1 where present."""
    import torch
    present = torch.empty(num_cols, dtype=torch.uint8, device=d_cols.device)
    call("dsp_col_presence", d_cols.data_ptr(), d_cols.numel(), num_cols, present.data_ptr(), stream)
    return present


def tile_device(d_cols, num_cols: int, T: int, present=None, stream: int = 0) -> Tiling:
    """tile() computed on the GPU from the local column ids already in device memory (a
    CUDA int64 tensor); `present` (their col_presence map) is reused when given."""
    cpt = c_i64()
    n_col = np.zeros(T, np.int32)
    n_slice = np.zeros(T, np.int32)
    nnz = np.zeros(T, np.int64)
    off = np.zeros(T + 1, np.int64)
    pp = present.data_ptr() if present is not None else None
    call("dsp_tile_device", d_cols.data_ptr(), d_cols.numel(), pp, num_cols, T, ctypes.byref(cpt), _ptr(n_col, c_i32),
         _ptr(n_slice, c_i32), _ptr(nnz, c_i64), _ptr(off, c_i64), None, stream)
    needed = np.zeros(max(int(off[-1]), 1), np.int32)
    call("dsp_tile_device", d_cols.data_ptr(), d_cols.numel(), pp, num_cols, T, None, None, None, None,
         _ptr(off, c_i64), _ptr(needed, c_i32), stream)
    return Tiling(int(cpt.value), n_col, n_slice, nnz, off, needed[: int(off[-1])])


def needed_from_presence(present, num_cols: int, T: int, stream: int = 0):
    """(n_col, offsets, ascending tile-local lists) of a device presence map; with the
    element-wise max of the ranks' maps this is the node union of merge_needed."""
    n_col = np.zeros(T, np.int32)
    off = np.zeros(T + 1, np.int64)
    call("dsp_tile_device", None, 0, present.data_ptr(), num_cols, T, None, _ptr(n_col, c_i32), None, None,
         _ptr(off, c_i64), None, stream)
    cols = np.zeros(max(int(off[-1]), 1), np.int32)
    call("dsp_tile_device", None, 0, present.data_ptr(), num_cols, T, None, None, None, None, _ptr(off, c_i64),
         _ptr(cols, c_i32), stream)
    return n_col, off, cols[: int(off[-1])]


def hierarchical_iterative_refinement_allocation(demand, node_of_gpu, tasks_per_gpu: int,
                                                 max_inter_node_iterations: int = 5,
                                                 max_intra_node_iterations: int = 5) -> np.ndarray:
    """HSDMA: remap[T] = owner rank of each tile from the P x T demand matrix."""
    D = _i32(demand)
    Pn, T = D.shape
    nodes = _i32(node_of_gpu)
    remap = np.zeros(T, np.int32)
    call("dsp_hsdma", _ptr(D, c_i32), Pn, T, _ptr(nodes, c_i32), tasks_per_gpu, max_inter_node_iterations,
         max_intra_node_iterations, _ptr(remap, c_i32))
    return remap


hsdma = hierarchical_iterative_refinement_allocation


def alloc_slice(P_: int, n_rolls: int) -> np.ndarray:
    r = np.zeros(P_ * n_rolls, np.int32)
    call("dsp_alloc_slice", P_, n_rolls, _ptr(r, c_i32))
    return r


def alloc_random(P_: int, n_rolls: int, seed: int = 0x5EED) -> np.ndarray:
    r = np.zeros(P_ * n_rolls, np.int32)
    call("dsp_alloc_random", P_, n_rolls, seed, _ptr(r, c_i32))
    return r


def allocate(task_dist: int, demand, n_rolls: int, node_of_gpu=None) -> np.ndarray:
    """The task_dist switch of src/dist_spmm_node.cu:137-158."""
    D = _i32(demand)
    Pn = D.shape[0]
    if task_dist == 0:
        return alloc_slice(Pn, n_rolls)
    if task_dist == 1:
        return alloc_random(Pn, n_rolls)
    if task_dist == 2:
        nodes = np.zeros(Pn, np.int32) if node_of_gpu is None else node_of_gpu
        return hsdma(D, nodes, n_rolls)
    raise ValueError("Wrong task distribution type.")


def merge_needed(counts, cols):
    """Union of R ranks' needed sets per tile (counts R x T, cols flat rank-major).
    Returns (n_col_merged int32[T], offsets int64[T+1], merged int32 flat)."""
    counts = _i32(counts)
    R, T = counts.shape
    cols = _i32(cols) if np.size(cols) else np.zeros(1, np.int32)
    off = np.zeros(T + 1, np.int64)
    n = np.zeros(T, np.int32)
    call("dsp_merge_needed", R, T, _ptr(counts, c_i32), _ptr(cols, c_i32), _ptr(off, c_i64), None, _ptr(n, c_i32))
    merged = np.zeros(max(int(off[-1]), 1), np.int32)
    call("dsp_merge_needed", R, T, _ptr(counts, c_i32), _ptr(cols, c_i32), _ptr(off, c_i64), _ptr(merged, c_i32),
         _ptr(n, c_i32))
    return n, off, merged[: int(off[-1])]


def comm_model_preset(platform="h100", tier: int = 0):
    m = dsp_comm_model()
    call("dsp_comm_model_preset", PLATFORM.get(platform, platform), tier, ctypes.byref(m))
    return m


def comm_select(comm_type: int, dims: int, n_col, n_slice, platform="h100", with_inter: bool = False):
    """Per-tile sparse (1) / bulk (0) decisions; returns intra (and inter) uint8 arrays."""
    n_col = _i32(n_col)
    n_slice = _i32(n_slice)
    T = n_col.shape[0]
    intra = comm_model_preset(platform, 0)
    inter = comm_model_preset(platform, 1)
    si = np.zeros(T, np.uint8)
    se = np.zeros(T, np.uint8)
    call("dsp_comm_select", comm_type, dims, ctypes.byref(intra), ctypes.byref(inter), T, _ptr(n_col, c_i32),
         _ptr(n_slice, c_i32), si.ctypes.data_as(_u8p), se.ctypes.data_as(_u8p) if with_inter else None)
    return (si, se) if with_inter else si


def traffic_intra(me: int, remap, sparse, n_col, n_slice, dims: int) -> int:
    remap, n_col, n_slice = _i32(remap), _i32(n_col), _i32(n_slice)
    sparse = np.ascontiguousarray(sparse, np.uint8)
    b = c_i64()
    call("dsp_traffic_intra", me, remap.shape[0], _ptr(remap, c_i32), sparse.ctypes.data_as(_u8p),
         _ptr(n_col, c_i32), _ptr(n_slice, c_i32), dims, ctypes.byref(b))
    return int(b.value)


def traffic_inter(me: int, ranks_per_node: int, num_nodes: int, remap, sparse_inter, n_col, n_slice,
                  dims: int) -> int:
    remap, n_col, n_slice = _i32(remap), _i32(n_col), _i32(n_slice)
    sp = np.ascontiguousarray(sparse_inter, np.uint8)
    b = c_i64()
    call("dsp_traffic_inter", me, ranks_per_node, num_nodes, remap.shape[0], _ptr(remap, c_i32),
         sp.ctypes.data_as(_u8p), _ptr(n_col, c_i32), _ptr(n_slice, c_i32), dims, ctypes.byref(b))
    return int(b.value)


def gflops(nnz: int, dims: int, avg_ms: float) -> float:
    return float(lib().dsp_gflops(nnz, dims, avg_ms))
