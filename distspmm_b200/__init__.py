"""distspmm_b200 — B200-native distributed CSR x dense SpMM (the hot path of DistSpMM).

Layers
  include/distspmm.h        C ABI (the drop-in boundary)
  libdistspmm_b200.so       native library: loader, planner, sm_100a kernels, rank runtime
  bin/dist_spmm_node        reference-compatible CLI
  matrix / planner / spmm / dist   Python face of the C ABI (ctypes; torch only supplies
                            device memory, streams and torch.distributed)
  comm_test / fit_comm_model       the bulk-vs-sparse fetch microbenchmark and the
                            selector-model fit (command lines of the reference's tools)
"""
from ._lib import DspError, lib
from .matrix import Csr, dense_b, dense_b_rows, gen_rmat, gen_stencil27, gen_uniform, load_from_csr, load_rows, make_matrix, save_csr
from . import planner
from .planner import hierarchical_iterative_refinement_allocation

__all__ = [
    "DspError", "lib", "Csr", "dense_b", "dense_b_rows", "gen_rmat", "gen_stencil27", "gen_uniform", "load_from_csr", "load_rows",
    "make_matrix", "save_csr", "planner", "hierarchical_iterative_refinement_allocation",
]


def __getattr__(name):
    # torch-dependent modules load on first use
    if name in ("SpmmPlan",):
        from .spmm import SpmmPlan
        return SpmmPlan
    if name in ("Rank", "build_local_group", "TorchComm", "distributed_plan", "connect_peers", "make_rank",
                "global_plan", "fetch_view"):
        from . import dist
        return getattr(dist, name)
    raise AttributeError(name)
