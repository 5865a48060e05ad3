"""Generate the golden fixtures of tests/golden/ (run where the reference checkout exists).

    DSP_REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py

Fixtures and their source of truth:
  hsdma_cases.json     remap[] from the reference's own hierarchical_iterative_refinement_
                       allocation (src/h_sdma.h:78-228) compiled from the reference sources
                       (oracle/_ref/libdsp_ref.so), on seeded random demand matrices.
  csr_small_*.bin      a small binary CSR (R-MAT scale 9) in the reference's file format;
  csr_small_ref.json   what the reference loader (src/sparse_matrix.h:83-159) and
                       turn_local_l_u_csr (:178-199) return for it (whole matrix and the
                       rows of every rank at P = 3), as arrays.
  thresholds.json      the adaptive-selector threshold 1/(a*pow(k,u)+b/k) of
                       src/comm_man.h:396-400 evaluated by an nvcc-compiled probe
                       (oracle/threshold_probe.cu), bit patterns, for the H100 and A800
                       constants and dims 1..2048.
  merge_cases.json     the node union of the ranks' needed sets from the reference's own
                       double_level_comm_node_processing (src/utils.h:439-547), compiled
                       with the thread-rank MPI stand-in (oracle/_ref/libdsp_ref_mpi.so) and
                       run with one thread per rank: inputs (per-rank counts and lists of
                       small R-MAT / stencil / uniform tilings) and the merged counts and
                       ascending lists.
  hsdma_mpi_cases.json remap[] every rank holds after the reference's ComputeAllocation_
                       HSDMA_MPI (src/utils.h:358-437), same build, seeded random demands.
  comm_model_fit.json  the reference's own model fit (tools/fit_comm_model.py, imported
                       from the reference tree): the (dims, mean critical density) inputs
                       it fits per tier and the (a, b, c, u) it returns.
Nothing here runs on the GPU box; the tests only read the committed files.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

DIMS = [1, 2, 3, 4, 7, 8, 16, 32, 47, 48, 64, 100, 105, 106, 128, 256, 512, 1024, 2048]


def make_hsdma():
    rng = np.random.default_rng(20240601)
    cases = []
    for i in range(60):
        P = int(rng.choice([1, 2, 3, 4, 8, 16]))
        nodes = int(rng.choice([n for n in (1, 2, 4) if P % n == 0]))
        rolls = int(rng.integers(1, 5))
        T = P * rolls
        hi = int(rng.choice([3, 50, 40000]))
        D = rng.integers(0, hi, size=(P, T)).astype(np.int32)
        node = np.repeat(np.arange(nodes), P // nodes).astype(np.int32)
        it = (5, 5) if i % 7 else (int(rng.integers(0, 4)), int(rng.integers(0, 8)))
        remap = oracle.hsdma(D, node, rolls, it[0], it[1], use_ref=True)
        cases.append(dict(demand=D.tolist(), node_of_gpu=node.tolist(), tasks_per_gpu=rolls,
                          max_inter=it[0], max_intra=it[1], remap=remap.tolist()))
    with open(os.path.join(HERE, "hsdma_cases.json"), "w") as f:
        json.dump(cases, f)


def make_merge():
    import distspmm_b200 as d
    from distspmm_b200 import planner
    cases = []
    mats = [("rmat10", d.gen_rmat(10, seed=11)), ("stencil6", d.gen_stencil27(6, seed=12)),
            ("uniform600x5", d.gen_uniform(600, 5, seed=13))]
    for name, A in mats:
        for P, rolls in ((2, 4), (3, 2), (4, 1), (8, 4)):
            T = P * rolls
            tilings = [planner.tile(planner.partition(A, *planner.bounds(A, P, p, "rows")), T) for p in range(P)]
            counts = np.stack([t.n_col for t in tilings]).astype(np.int32)
            flat = np.concatenate([t.needed for t in tilings]).astype(np.int32)
            n, off, merged = oracle.ref_node_merge(counts, flat)
            cases.append(dict(matrix=name, P=P, n_rolls=rolls, cpt=int(tilings[0].cpt), counts=counts.tolist(),
                              lists=flat.tolist(), merged_count=n.tolist(), offsets=off.tolist(),
                              merged=merged.tolist()))
    with open(os.path.join(HERE, "merge_cases.json"), "w") as f:
        json.dump(cases, f)


def make_hsdma_mpi():
    rng = np.random.default_rng(20240602)
    cases = []
    for _ in range(24):
        P = int(rng.choice([1, 2, 3, 4, 8]))
        nodes = int(rng.choice([n for n in (1, 2, 4) if P % n == 0]))
        rolls = int(rng.integers(1, 5))
        T = P * rolls
        D = rng.integers(0, int(rng.choice([3, 60, 50000])), size=(P, T)).astype(np.int32)
        node = np.repeat(np.arange(nodes), P // nodes).astype(np.int32)
        remap = oracle.ref_hsdma_mpi(D, node, rolls)
        assert (remap == remap[0]).all()
        cases.append(dict(demand=D.tolist(), node_of_gpu=node.tolist(), tasks_per_gpu=rolls,
                          remap=remap[0].tolist()))
    with open(os.path.join(HERE, "hsdma_mpi_cases.json"), "w") as f:
        json.dump(cases, f)


def make_csr():
    import distspmm_b200 as d
    A = d.gen_rmat(9, 8, seed=7)
    prefix = os.path.join(HERE, "csr_small")
    d.save_csr(prefix, A)
    out = {"whole": None, "parts": []}
    whole = oracle.ref_load(prefix)
    out["whole"] = {k: (v.tolist() if isinstance(v, np.ndarray) else v) for k, v in whole.items()}
    M = whole["num_rows"]
    for r in range(3):
        lb, ub = oracle.partition_bounds(M, 3, r)
        part = oracle.ref_load(prefix, lb, ub)
        out["parts"].append({"lb": lb, "ub": ub, **{k: (v.tolist() if isinstance(v, np.ndarray) else v)
                                                     for k, v in part.items()}})
    with open(os.path.join(HERE, "csr_small_ref.json"), "w") as f:
        json.dump(out, f)


def make_thresholds():
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "probe")
        subprocess.run(["nvcc", "-O2", os.path.join(ROOT, "oracle", "threshold_probe.cu"), "-o", exe], check=True)
        res = {}
        for name, model in [("h100_intra", oracle.H100_INTRA), ("h100_inter", oracle.H100_INTER),
                            ("a800_intra", oracle.A800_INTRA), ("a800_inter", oracle.A800_INTER)]:
            # pass the float value of each constant exactly (repr of the float32)
            args = [repr(float(np.float32(x))) for x in model]
            r = subprocess.run([exe] + args + [str(x) for x in DIMS], check=True, capture_output=True, text=True)
            res[name] = {"model": [float(np.float32(x)) for x in model],
                         "thr_bits": {ln.split()[0]: ln.split()[1] for ln in r.stdout.strip().splitlines()}}
    with open(os.path.join(HERE, "thresholds.json"), "w") as f:
        json.dump(res, f, indent=1)


def make_fit(ref_root=None):
    ref_root = ref_root or os.environ["DSP_REFERENCE_ROOT"]
    import importlib.util
    spec = importlib.util.spec_from_file_location("ref_fit", os.path.join(ref_root, "tools", "fit_comm_model.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    params = ref.fit_all()
    group0 = [0, 2, 4, 6]  # the runs the reference averages before fitting (fit_all)
    out = {"dims": list(ref.DIMS)}
    for tier, col in (("intra", 1), ("inter", 2)):
        out[tier] = {"threshold": np.mean([ref.MEASURED[i][col] for i in group0], axis=0).tolist(),
                     "params": [float(x) for x in params[tier]]}
    with open(os.path.join(HERE, "comm_model_fit.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    make_fit()
    oracle.build(ref=True, ref_src=os.path.join(os.environ["DSP_REFERENCE_ROOT"], "src"))
    if oracle.ref_lib() is None or oracle.ref_mpi_lib() is None:
        sys.exit("reference shim not available: run where the reference sources exist")
    make_hsdma()
    make_merge()
    make_hsdma_mpi()
    make_csr()
    make_thresholds()
    print("golden fixtures written to", HERE)
