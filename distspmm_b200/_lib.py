"""ctypes binding of libdistspmm_b200.so (the C ABI declared in include/distspmm.h).

The library must exist: there is no Python or CPU fallback for any compute entry point.
Build it with ``python -m distspmm_b200.build``.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libdistspmm_b200.so")

c_i64 = ctypes.c_int64
c_i32 = ctypes.c_int32
c_int = ctypes.c_int
c_u64 = ctypes.c_uint64
c_f32 = ctypes.c_float
c_f64 = ctypes.c_double
c_vp = ctypes.c_void_p
P = ctypes.POINTER

DSP_OK = 0
ERRORS = {
    -1: "DSP_ERR_INVALID", -2: "DSP_ERR_IO", -3: "DSP_ERR_FORMAT", -4: "DSP_ERR_CUDA",
    -5: "DSP_ERR_NOMEM", -6: "DSP_ERR_UNSUPPORTED", -7: "DSP_ERR_TIMEOUT", -8: "DSP_ERR_STATE",
}
PLATFORM = {"h100": 0, "a800": 1, "b200": 2}


class DspError(RuntimeError):
    """A DSP_ERR_* status returned by the native library."""

    def __init__(self, code: int, where: str, msg: str):
        self.code = code
        super().__init__(f"{where}: {ERRORS.get(code, code)}: {msg}")


class dsp_csr(ctypes.Structure):
    _fields_ = [("num_rows", c_i64), ("num_cols", c_i64), ("nnz", c_i64),
                ("indptr", P(c_i64)), ("indices", P(c_i64)), ("values", P(c_f32))]


class dsp_comm_model(ctypes.Structure):
    _fields_ = [("a", c_f32), ("b", c_f32), ("c", c_f32), ("u", c_f32)]


class dsp_spmm_info(ctypes.Structure):
    _fields_ = [(n, c_i64) for n in ("rows", "cols", "nnz", "variant", "items", "split_rows", "pieces",
                                     "piece_cap", "max_row_len", "scratch_bytes", "device_bytes")]


class dsp_rank_desc(ctypes.Structure):
    _fields_ = [("rank", c_int), ("world", c_int), ("device", c_int), ("dims", c_int), ("T", c_int),
                ("n_streams", c_int), ("cpt", c_i64), ("M", c_i64), ("m_lb", c_i64),
                ("local", P(dsp_csr)), ("remap", P(c_i32)), ("sparse", P(ctypes.c_uint8)),
                ("needed_offsets", P(c_i64)), ("needed_cols", P(c_i32)), ("n_slice", P(c_i32)),
                ("fetch_engine", c_int), ("pipeline", c_int), ("groups", c_int)]


class dsp_rank_stats(ctypes.Structure):
    _fields_ = [(n, c_i64) for n in ("m_local", "nnz_local", "segments", "fetch_rows", "fetch_bytes",
                                     "fetch_bulk_tiles", "fetch_sparse_tiles", "owned_rows",
                                     "distinct_cols", "launches_per_step", "kernels_per_step",
                                     "device_bytes", "pipeline", "phase0_nnz", "timeline_len")] + [
        (n, ctypes.c_float) for n in ("model_rows_ms", "model_split_ms", "model_groups_ms")]


class dsp_args(ctypes.Structure):
    _fields_ = [("file", ctypes.c_char_p), ("matrix", P(dsp_csr)), ("dims", c_int), ("task_dist", c_int),
                ("comm_type", c_int), ("n_rolls", c_int), ("repeat", c_int), ("n_streams", c_int),
                ("world", c_int), ("devices", P(c_int)), ("platform", c_int), ("b_seed", c_u64),
                ("b_ones", c_int), ("c_out", P(c_f32))]


class dsp_report(ctypes.Structure):
    _fields_ = [("stage_ms", c_f64 * 8), ("hsdma_ms", c_f64), ("avg_ms", c_f64), ("min_ms", c_f64),
                ("median_ms", c_f64), ("reps_counted", c_int), ("traffic_intra", c_i64),
                ("traffic_inter", c_i64), ("fetched_bytes", c_i64), ("mem_gb", c_f64),
                ("gflops", c_f64), ("nnz", c_i64), ("M", c_i64), ("T", c_int), ("remap", c_i32 * 4096),
                ("row_lb", c_i64), ("row_ub", c_i64)]


# name -> (restype, argtypes); every status-returning function is checked by call().
PROTOTYPES = {
    "dsp_last_error": (ctypes.c_char_p, []),
    "dsp_version": (ctypes.c_char_p, []),
    "dsp_device_count": (c_int, []),
    "dsp_csr_load": (c_int, [ctypes.c_char_p, P(dsp_csr)]),
    "dsp_csr_load_rows": (c_int, [ctypes.c_char_p, c_i64, c_i64, P(dsp_csr)]),
    "dsp_csr_save": (c_int, [ctypes.c_char_p, P(dsp_csr)]),
    "dsp_csr_read_indptr": (c_int, [ctypes.c_char_p, P(c_i64), P(c_i64)]),
    "dsp_csr_alloc": (c_int, [c_i64, c_i64, c_i64, P(dsp_csr)]),
    "dsp_csr_free": (None, [P(dsp_csr)]),
    "dsp_csr_validate": (c_int, [P(dsp_csr)]),
    "dsp_gen_rmat": (c_int, [c_int, c_int, c_f64, c_f64, c_f64, c_u64, P(dsp_csr)]),
    "dsp_gen_stencil27": (c_int, [c_i64, c_u64, P(dsp_csr)]),
    "dsp_gen_uniform": (c_int, [c_i64, c_i64, c_u64, P(dsp_csr)]),
    "dsp_fill_dense_host": (c_int, [P(c_f32), c_i64, c_i64, c_i64, c_i64, c_u64]),
    "dsp_fill_dense_rows_host": (c_int, [P(c_f32), P(c_i64), c_i64, c_i64, c_i64, c_u64]),
    "dsp_partition_bounds": (c_int, [c_i64, c_int, c_int, P(c_i64), P(c_i64)]),
    "dsp_partition_bounds_balanced": (c_int, [P(c_i64), c_i64, c_int, c_int, P(c_i64), P(c_i64)]),
    "dsp_partition": (c_int, [P(dsp_csr), c_i64, c_i64, P(dsp_csr)]),
    "dsp_tile_counts": (c_int, [P(dsp_csr), c_int, P(c_i64), P(c_i32), P(c_i32), P(c_i64)]),
    "dsp_tile_needed": (c_int, [P(dsp_csr), c_int, P(c_i64), P(c_i32)]),
    "dsp_col_presence": (c_int, [c_vp, c_i64, c_i64, c_vp, c_vp]),
    "dsp_tile_device": (c_int, [c_vp, c_i64, c_vp, c_i64, c_int, P(c_i64), P(c_i32), P(c_i32), P(c_i64), P(c_i64),
                                P(c_i32), c_vp]),
    "dsp_hsdma": (c_int, [P(c_i32), c_int, c_int, P(c_i32), c_int, c_int, c_int, P(c_i32)]),
    "dsp_alloc_slice": (c_int, [c_int, c_int, P(c_i32)]),
    "dsp_alloc_random": (c_int, [c_int, c_int, c_u64, P(c_i32)]),
    "dsp_merge_needed": (c_int, [c_int, c_int, P(c_i32), P(c_i32), P(c_i64), P(c_i32), P(c_i32)]),
    "dsp_comm_model_preset": (c_int, [c_int, c_int, P(dsp_comm_model)]),
    "dsp_comm_select": (c_int, [c_int, c_int, P(dsp_comm_model), P(dsp_comm_model), c_int, P(c_i32),
                                P(c_i32), P(ctypes.c_uint8), P(ctypes.c_uint8)]),
    "dsp_traffic_intra": (c_int, [c_int, c_int, P(c_i32), P(ctypes.c_uint8), P(c_i32), P(c_i32), c_int,
                                  P(c_i64)]),
    "dsp_traffic_inter": (c_int, [c_int, c_int, c_int, c_int, P(c_i32), P(ctypes.c_uint8), P(c_i32),
                                  P(c_i32), c_int, P(c_i64)]),
    "dsp_gflops": (c_f64, [c_i64, c_int, c_f64]),
    "dsp_spmm_plan_create": (c_int, [c_int, P(dsp_csr), c_int, c_int, P(c_vp)]),
    "dsp_spmm_plan_destroy": (None, [c_vp]),
    "dsp_spmm_plan_info": (c_int, [c_vp, P(dsp_spmm_info)]),
    "dsp_spmm_f32": (c_int, [c_vp, c_vp, c_i64, c_vp, c_i64, c_int, c_int, c_vp]),
    "dsp_spmm_check_error": (c_int, [c_vp]),
    "dsp_spmm_csr_f32_noalloc": (c_int, [c_vp, c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_int,
                                         c_int, c_vp]),
    "dsp_rank_create": (c_int, [P(dsp_rank_desc), P(c_vp)]),
    "dsp_rank_destroy": (None, [c_vp]),
    "dsp_rank_stats_get": (c_int, [c_vp, P(dsp_rank_stats)]),
    "dsp_rank_b_ptr": (c_int, [c_vp, P(c_vp)]),
    "dsp_rank_c_ptr": (c_int, [c_vp, P(c_vp)]),
    "dsp_rank_ipc_handle": (c_int, [c_vp, c_vp]),
    "dsp_rank_open_peer": (c_int, [c_vp, c_int, c_vp]),
    "dsp_rank_set_peer": (c_int, [c_vp, c_int, c_vp, c_int]),
    "dsp_rank_fill_b": (c_int, [c_vp, c_u64, c_vp]),
    "dsp_rank_upload_b": (c_int, [c_vp, c_vp, c_vp]),
    "dsp_rank_upload_b_owned": (c_int, [c_vp, c_vp, c_vp]),
    "dsp_rank_poison_remote": (c_int, [c_vp, c_vp]),
    "dsp_rank_step": (c_int, [c_vp, c_vp]),
    "dsp_rank_check_error": (c_int, [c_vp]),
    "dsp_selftest_bounded_wait": (c_int, [ctypes.c_longlong, P(c_int)]),
    "dsp_comm_probe": (c_int, [c_int, c_int, c_i64, c_int, P(c_i32), c_int, P(c_i64), c_int, c_int, P(c_f64),
                               P(c_f64)]),
    "dsp_rank_download_c": (c_int, [c_vp, c_vp, c_vp]),
    "dsp_rank_last_compute_ms": (c_int, [c_vp, P(c_f32)]),
    "dsp_rank_last_timeline": (c_int, [c_vp, P(c_f32), c_int]),
    "dsp_run": (c_int, [P(dsp_args), P(dsp_report)]),
    "dsp_store_open": (c_int, [ctypes.c_char_p, c_int, c_int, c_f64, P(c_vp)]),
    "dsp_store_allgather": (c_int, [c_vp, ctypes.c_char_p, c_vp, c_i64, c_vp, c_i64, P(c_i64)]),
    "dsp_store_barrier": (c_int, [c_vp, ctypes.c_char_p]),
    "dsp_store_close": (None, [c_vp, c_int]),
    "dsp_run_rank": (c_int, [P(dsp_args), c_int, c_int, c_int, c_vp, P(dsp_report)]),
}

_lib = None


def lib():
    """Load the native library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m distspmm_b200.build` "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call a status-returning entry point; raise DspError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != DSP_OK:
        raise DspError(rc, name, lib().dsp_last_error().decode(errors="replace"))
