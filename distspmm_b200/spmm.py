"""Single-GPU SpMM through the native sm_100a kernels.

``SpmmPlan`` holds A on the device (work items, int32 columns, fp32 values) and runs
C = A.B / C += A.B on torch tensors (device memory and streams come from torch; the
arithmetic is the library's). It is the drop-in for the per-tile
cusparseCreateCoo + cusparseSpMM of src/dist_spmm_node.cu:233-234, :354-385.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import c_vp, call, dsp_spmm_info, lib
from .matrix import Csr


class SpmmPlan:
    VARIANTS = {None: -1, "auto": -1, "rows": 0, "nnz": 1}

    def __init__(self, a: Csr, device: int = 0, dims_hint: int = 128, variant: str | None = None):
        self.device = device
        self.rows = a.num_rows
        self.cols = a.num_cols
        self.nnz = a.nnz
        c = a.to_c()
        h = c_vp()
        call("dsp_spmm_plan_create", device, ctypes.byref(c), dims_hint, self.VARIANTS[variant], ctypes.byref(h))
        self._h = h

    def info(self) -> dict:
        i = dsp_spmm_info()
        call("dsp_spmm_plan_info", self._h, ctypes.byref(i))
        return {k: int(getattr(i, k)) for k, _ in dsp_spmm_info._fields_}

    def run_ptr(self, B_ptr: int, ldb: int, C_ptr: int, ldc: int, N: int, accumulate: bool = False,
                stream: int = 0) -> None:
        """Raw-pointer form of the C ABI call (device pointers, cudaStream_t as int)."""
        call("dsp_spmm_f32", self._h, B_ptr, ldb, C_ptr, ldc, N, int(accumulate), stream)

    def __call__(self, B: torch.Tensor, C: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
        assert B.is_cuda and B.dtype == torch.float32 and B.dim() == 2 and B.stride(1) == 1
        assert B.shape[0] == self.cols, f"B has {B.shape[0]} rows, A has {self.cols} columns"
        N = B.shape[1]
        if C is None:
            C = torch.empty((self.rows, N), dtype=torch.float32, device=B.device)
        assert C.is_cuda and C.dtype == torch.float32 and C.stride(1) == 1 and tuple(C.shape) == (self.rows, N)
        stream = torch.cuda.current_stream(B.device).cuda_stream
        self.run_ptr(B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0), N, accumulate, stream)
        return C

    def check_error(self) -> None:
        """After the stream was synchronised: raise DspError if a kernel's bounded wait on its
        staged copies gave up (the flag is cleared)."""
        call("dsp_spmm_check_error", self._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dsp_spmm_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
