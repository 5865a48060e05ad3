"""Build recipe of the native library (sm_100a) and the CLI drivers.

    python -m distspmm_b200.build            # incremental
    python -m distspmm_b200.build --force    # rebuild everything

Outputs (in-tree, git-ignored, shipped with the source snapshot to the GPU box):
    distspmm_b200/libdistspmm_b200.so   the C-ABI library (include/distspmm.h)
    distspmm_b200/bin/dist_spmm_node    the reference-compatible CLI
    distspmm_b200/bin/dist_spmm         alias CLI (single-node, same pipeline)
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdistspmm_b200.so")
BIN = os.path.join(PKG, "bin")

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-ffp-contract=off",
                     "-I" + os.path.join(ROOT, "include")]
CXX = os.environ.get("CXX", "g++")
CXX_FLAGS = ["-O3", "-fPIC", "-std=c++17", "-ffp-contract=off", "-pthread", "-Wall",
             "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(os.path.dirname(NVCC), "..", "include")]

CU_SOURCES = ["spmm.cu", "rank.cu", "fetch.cu", "setup.cu"]
CPP_SOURCES = ["host_csr.cpp", "host_gen.cpp", "host_plan.cpp", "run.cpp", "run_rank.cpp", "store.cpp"]
HEADERS = ["common.h", "internal.h", "device.cuh"]
CLI_SOURCES = {"dist_spmm_node": "cli_dist_spmm_node.cpp"}


def _newer(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(BIN, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "distspmm.h")]
    jobs = []
    objs = []
    for s in CU_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJ, s + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + hdrs):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([NVCC] + NVCC_FLAGS + extra + ["-c", src, "-o", obj])
    for s in CPP_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(OBJ, s + ".o")
        objs.append(obj)
        if force or _newer(obj, [src] + hdrs):
            jobs.append([CXX] + CXX_FLAGS + ["-c", src, "-o", obj])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for out in ex.map(_run, jobs):
            logs.append(out)
    if force or jobs or not os.path.exists(LIB):
        logs.append(_run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs +
                         ["-Xlinker", "-z,defs", "-lpthread", "-lrt", "-ldl"]))
    for name, src in CLI_SOURCES.items():
        src = os.path.join(CSRC, src)
        out = os.path.join(BIN, name)
        if force or _newer(out, [src, LIB] + hdrs):
            logs.append(_run([CXX] + CXX_FLAGS + [src, "-o", out, "-L" + PKG, "-ldistspmm_b200",
                              "-Wl,-rpath,$ORIGIN/.."]))
    alias = os.path.join(BIN, "dist_spmm")
    if os.path.exists(os.path.join(BIN, "dist_spmm_node")):
        if os.path.lexists(alias):
            os.remove(alias)
        os.symlink("dist_spmm_node", alias)
    text = "\n".join(x for x in logs if x)
    if verbose and text:
        print(text)
    return text


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v (registers, spills)")
    a = ap.parse_args(argv)
    out = build(force=a.force or a.ptxas_info, verbose=True, ptxas_info=a.ptxas_info)
    print("built", LIB)
    return 0


if __name__ == "__main__":
    sys.exit(main())
