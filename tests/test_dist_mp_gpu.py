"""The one-process-per-GPU path: ranks in separate processes (NCCL host collectives,
CUDA IPC for the peers' B buffers, NVLink fetches), each on its own GPU. The gathered C
must match the oracle; remote rows are NaN-poisoned before the step. Skipped when fewer
than 2 GPUs are visible."""
import os
import socket
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, comm_type, dims, device_setup=False):
    import datetime

    import torch
    import torch.distributed as dist

    import distspmm_b200 as d
    from distspmm_b200 import planner
    from distspmm_b200.dist import TorchComm, connect_peers, distributed_plan, make_rank

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    comm = TorchComm()
    A = d.gen_rmat(14, seed=5)
    lb, ub = planner.partition_bounds(A.num_rows, world, rank)
    local = planner.partition(A, lb, ub)
    tiling, plan = distributed_plan(comm, local, 4, 2)
    if device_setup:  # the GPU set-up path must agree with the host planner exactly
        t2, p2 = distributed_plan(comm, local, 4, 2, device_setup=True)
        for f in ("n_col", "n_slice", "nnz", "offsets", "needed"):
            assert np.array_equal(getattr(t2, f), getattr(tiling, f)), f
        for f in ("remap", "n_col", "offsets", "merged", "demand"):
            assert np.array_equal(getattr(p2, f), getattr(plan, f)), f
        tiling, plan = t2, p2
    R = make_rank(local, rank, world, rank, dims, A.num_rows, lb, tiling, plan, comm_type)
    connect_peers(comm, R)
    for it in range(2):
        R.poison_remote()
        R.fill_b(21 + it)
        torch.cuda.synchronize()
        comm.barrier()
        R.step()
        torch.cuda.synchronize()
        comm.barrier()
    C = np.empty((ub - lb, dims), np.float32)
    R.download_c(C)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"c{rank}.npy"), C)
    st = R.stats()
    np.save(os.path.join(out_dir, f"s{rank}.npy"), np.array([st["fetch_rows"], st["fetch_bytes"]]))
    comm.barrier()
    R.close()
    comm.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("comm_type,dims,device_setup", [(2, 128, False), (0, 64, False), (1, 32, False),
                                                        (2, 128, True)])
def test_two_process_pipeline(gpu, comm_type, dims, device_setup):
    import torch
    import torch.multiprocessing as mp

    import distspmm_b200 as d
    import oracle
    world = torch.cuda.device_count()
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(world, 4)
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_worker, args=(world, _free_port(), tmp, comm_type, dims, device_setup), nprocs=world,
                           start_method="spawn", join=True)
        A = d.gen_rmat(14, seed=5)
        C = np.concatenate([np.load(os.path.join(tmp, f"c{r}.npy")) for r in range(world)])
        fetched = sum(int(np.load(os.path.join(tmp, f"s{r}.npy"))[0]) for r in range(world))
    assert fetched > 0
    B = d.dense_b(A.num_cols, dims, seed=22)
    ref, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    assert np.isfinite(C).all(), "a remote row was used before it was fetched"
    ok, worst = oracle.check_close(C, ref, ab, 1e-5)
    assert ok, worst
