"""Comparison arms timed beside the engine (not part of the engine).

``CusparseArm`` runs the reference's local SpMM — cuSPARSE per-tile COO with int64
indices, fp32, CUSPARSE_SPMM_ALG_DEFAULT, beta = 1 over the column tiles
(src/dist_spmm_node.cu:206-234, :354-385) — and the whole local matrix as one CSR
SpMM, on device buffers the caller owns. ``build()`` compiles ``libdsp_cusparse.so``
next to this file.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "cusparse_arm.cu")
LIB = os.path.join(HERE, "libdsp_cusparse.so")
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-o", LIB, SRC, "-lcusparse"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("cuSPARSE arm build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return LIB


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise RuntimeError(f"{LIB} is missing: run baseline.build()")
        L = ctypes.CDLL(LIB)
        i64, vp = ctypes.c_int64, ctypes.c_void_p
        L.csa_create.argtypes = [i64, i64, vp, vp, vp, ctypes.c_int, ctypes.c_int, vp, vp, ctypes.POINTER(vp)]
        L.csa_run_tiles.argtypes = [vp, vp, vp, vp]
        L.csa_run_csr.argtypes = [vp, vp, vp, vp]
        L.csa_destroy.argtypes = [vp]
        L.csa_device_bytes.argtypes = [vp]
        L.csa_device_bytes.restype = i64
        L.csa_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


class CusparseArm:
    """cuSPARSE SpMM of a local CSR (host numpy arrays) against device B [M x dims] and
    C [m x dims] (torch CUDA tensors or raw device pointers)."""

    def __init__(self, local, M: int, T: int, dims: int, B_ptr: int, C_ptr: int):
        L = _load()
        self.h = ctypes.c_void_p()
        rc = L.csa_create(local.num_rows, M, local.indptr.ctypes.data, local.indices.ctypes.data,
                          local.values.ctypes.data, T, dims, B_ptr, C_ptr, ctypes.byref(self.h))
        if rc != 0:
            msg = L.csa_last_error().decode()
            self.close()
            raise RuntimeError(f"cuSPARSE arm set-up: {msg}")
        self.device_bytes = L.csa_device_bytes(self.h)

    def run_tiles(self, B_ptr: int, C_ptr: int, stream: int) -> None:
        if _load().csa_run_tiles(self.h, B_ptr, C_ptr, stream) != 0:
            raise RuntimeError(_load().csa_last_error().decode())

    def run_csr(self, B_ptr: int, C_ptr: int, stream: int) -> None:
        if _load().csa_run_csr(self.h, B_ptr, C_ptr, stream) != 0:
            raise RuntimeError(_load().csa_last_error().decode())

    def close(self) -> None:
        if self.h:
            _load().csa_destroy(self.h)
            self.h = ctypes.c_void_p()
