"""`mpirun -np P dist_spmm_node ...` as the reference is launched: one process per rank,
rank / world / local rank from the launcher's environment (here torchrun's and Open MPI's
variable names, set by the test), each process on the GPU of its local rank modulo the
visible GPUs, peers' B opened by CUDA IPC, host collectives through the store directory.
Each rank writes its rows of C (DSP_C_OUT); together they must match the oracle, and
rank 0's report must carry the same allocation and traffic lines as the single-process
`-np P` run of the same matrix."""
import os
import subprocess

import numpy as np
import pytest

import distspmm_b200 as d
import oracle

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _launch(exe, args, world, tmp, env_style, extra=None):
    procs = []
    for r in range(world):
        env = dict(os.environ, DSP_STORE_DIR=str(tmp / "store"), DSP_B_SEED="7", DSP_C_OUT=str(tmp / "c"),
                   DSP_STORE_TIMEOUT_S="120", **(extra or {}))
        for k in ("DSP_NP", "RANK", "WORLD_SIZE", "LOCAL_RANK", "OMPI_COMM_WORLD_RANK", "OMPI_COMM_WORLD_SIZE",
                  "OMPI_COMM_WORLD_LOCAL_RANK", "PMI_RANK", "PMI_SIZE", "SLURM_PROCID", "SLURM_NTASKS"):
            env.pop(k, None)
        if env_style == "torchrun":
            env.update(RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r))
        else:
            env.update(OMPI_COMM_WORLD_RANK=str(r), OMPI_COMM_WORLD_SIZE=str(world),
                       OMPI_COMM_WORLD_LOCAL_RANK=str(r))
        procs.append(subprocess.Popen([exe] + args, env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                                      text=True))
    outs = []
    for p in procs:
        try:
            o, e = p.communicate(timeout=300)
        except subprocess.TimeoutExpired:
            for q in procs:
                q.kill()
            raise
        outs.append((p.returncode, o, e))
    return outs


@pytest.mark.parametrize("world,env_style,extra", [
    (2, "torchrun", None),
    (3, "ompi", {"DSP_PARTITION": "balanced", "DSP_FETCH_SCOPE": "rank"}),
])
def test_cli_one_process_per_rank_matches_oracle(gpu, tmp_path, world, env_style, extra):
    from distspmm_b200 import build
    A = d.gen_rmat(12, seed=3)
    dims = 64
    prefix = str(tmp_path / "g")
    d.save_csr(prefix, A)
    exe = os.path.join(build.BIN, "dist_spmm_node")
    args = [prefix, str(dims), "2", "2", "2", "7", "4"]
    outs = _launch(exe, args, world, tmp_path, env_style, extra)
    for r, (rc, o, e) in enumerate(outs):
        assert rc == 0, f"rank {r}: {e[-2000:]}"
        assert (o.strip() != "") == (r == 0), "only rank 0 prints the report"
    assert not os.path.exists(tmp_path / "store"), "rank 0 removes the store directory"

    B = d.dense_b(A.num_cols, dims, 7)
    ref, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    parts = [np.fromfile(str(tmp_path / f"c.{r}"), np.float32).reshape(-1, dims) for r in range(world)]
    C = np.concatenate(parts)
    assert C.shape == (A.num_rows, dims)
    ok, worst = oracle.check_close(C, ref, ab, RTOL)
    assert ok, worst

    # the same allocation and traffic as the single-process run with -np P
    env = dict(os.environ, DSP_B_SEED="7", **(extra or {}))
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "OMPI_COMM_WORLD_RANK", "OMPI_COMM_WORLD_SIZE"):
        env.pop(k, None)
    single = subprocess.run([exe, "-np", str(world)] + args, env=env, capture_output=True, text=True, timeout=300)
    assert single.returncode == 0, single.stderr
    mp_lines = outs[0][1].strip().splitlines()
    sp_lines = single.stdout.strip().splitlines()
    assert mp_lines[:3] == sp_lines[:3]  # task distribution, remap, "Running ..." lines
    pick = lambda ls: [ln for ln in ls if ln.startswith("Communication Traffic")]  # noqa: E731
    assert pick(mp_lines) == pick(sp_lines)


def test_cli_rank_that_never_starts_is_reported(gpu, tmp_path):
    """Failure detection on the host: rank 1 of 2 never starts; rank 0 gives up after the
    store's bounded wait with an error instead of hanging."""
    from distspmm_b200 import build
    A = d.gen_rmat(9, seed=3)
    prefix = str(tmp_path / "g")
    d.save_csr(prefix, A)
    exe = os.path.join(build.BIN, "dist_spmm_node")
    env = dict(os.environ, DSP_STORE_DIR=str(tmp_path / "store"), DSP_STORE_TIMEOUT_S="2", RANK="0",
               WORLD_SIZE="2", LOCAL_RANK="0")
    env.pop("DSP_NP", None)
    r = subprocess.run([exe, prefix, "32", "2", "2", "2", "3"], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode != 0
    assert "rank gone or not started" in r.stderr
