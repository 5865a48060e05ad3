"""Bulk-vs-sparse fetch microbenchmark: the reference's comm_test (src/comm_test.cu:27-147)
on this engine's fetch paths.

    python -m distspmm_b200.comm_test <N> <dims_s> <dims_e> <stride> <gpu_shift> <bins> <com_type> \
        [--engine lsu|tma] [--reps R] [--json out.json]

For dims = dims_s, dims_s*stride, ... <= dims_e, GPU 0 times one copy-engine copy of the
whole N x dims fp32 buffer of its peer GPU (gpu_shift away; the bulk tile fetch) and the
gather kernel moving the first i*N/bins rows of a random permutation (i = 1..bins; the
sparse fetch), then prints ``<dims>,<threshold>`` as the reference does: threshold =
(i-1)/(bins+1) for the first i at which the sparse fetch is no faster than the bulk copy.
com_type 0 is the intra-node (NVLink) tier; 1, the inter-node tier, needs a second node and
is refused. Times are CUDA-event device times (the reference uses host wall clock around a
stream synchronise).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import sys

import numpy as np

from ._lib import P, c_f64, c_i32, c_i64, call
from .dist import FETCH_ENGINES


def probe(device: int, peer: int, rows: int, dims: int, row_ids: np.ndarray, counts, engine: str = "lsu",
          reps: int = 3):
    """(bulk_ms, [sparse_ms per count]) from dsp_comm_probe."""
    ids = np.ascontiguousarray(row_ids, np.int32)
    cnt = np.ascontiguousarray(counts, np.int64)
    out = np.zeros(max(cnt.size, 1), np.float64)
    bulk = c_f64()
    call("dsp_comm_probe", device, peer, rows, dims, ids.ctypes.data_as(P(c_i32)), int(cnt.size),
         cnt.ctypes.data_as(P(c_i64)), FETCH_ENGINES[engine], reps, ctypes.byref(bulk),
         out.ctypes.data_as(P(c_f64)))
    return float(bulk.value), out[: cnt.size].tolist()


def critical_density(bulk_ms: float, sparse_ms, bins: int) -> float:
    """The reference's threshold: (i-1)/(bins+1), i the first density index (1-based) whose
    sparse time is not below the bulk time (bins+1 when the sparse fetch always wins)."""
    i = 1
    while i < bins + 1 and bulk_ms > sparse_ms[i - 1]:
        i += 1
    return (i - 1) / (bins + 1)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    for name in ("N", "dims_s", "dims_e", "stride", "gpu_shift", "bins", "com_type"):
        ap.add_argument(name, type=int)
    ap.add_argument("--engine", choices=sorted(FETCH_ENGINES), default="lsu")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--json", help="write dims, thresholds and raw times here")
    a = ap.parse_args(argv)
    if a.com_type != 0:
        print("inter-node tier (com_type 1): needs a second node; this build measures one node", file=sys.stderr)
        return 2
    if a.N < 1 or a.dims_s < 1 or a.stride < 2 or a.bins < 1:
        print("N, dims_s >= 1, stride >= 2, bins >= 1", file=sys.stderr)
        return 2
    from ._lib import lib
    ngpu = lib().dsp_device_count()
    if ngpu < 1:
        print("no CUDA device", file=sys.stderr)
        return 2
    peer = max(1, a.gpu_shift) % ngpu
    if peer == 0:
        print(f"note: one visible GPU; measuring a local copy (peer = device 0)", file=sys.stderr)
    perm = np.random.default_rng(a.seed).permutation(a.N).astype(np.int32)
    counts = [int(a.N * (i / a.bins)) for i in range(1, a.bins + 1)]
    print(f"comm buffer size of send and recv : {a.N * a.dims_e * 4 / 2**30:.3f} GiB")
    print("Communication type: intra node communication")
    res = {"N": a.N, "bins": a.bins, "engine": a.engine, "peer": peer, "dims": [], "threshold": [], "bulk_ms": [],
           "sparse_ms": []}
    dims = a.dims_s
    while dims <= a.dims_e:
        bulk, sparse = probe(0, peer, a.N, dims, perm, counts, a.engine, a.reps)
        thr = critical_density(bulk, sparse, a.bins)
        print(f"Dim: {dims} Comm-size: {a.N * dims * 4 / 2**30:.3f} GiB message size: {dims * 4} B")
        print("========================== ")
        print(f"{dims},{thr}")
        res["dims"].append(dims)
        res["threshold"].append(thr)
        res["bulk_ms"].append(bulk)
        res["sparse_ms"].append(sparse)
        dims *= a.stride
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f)
    return 0


if __name__ == "__main__":
    sys.exit(main())
