"""The host collectives of the distributed setup, run as 2 (and 3) gloo ranks on the CPU:
every rank's TorchComm-driven plan (demand all-gather, allocation, needed-set merge) must
equal the plan computed in one process from all ranks' tilings. Also the failure path: a
rank that never joins makes the others' collectives time out with an error."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir, task_dist, partition="rows"):
    import datetime

    import torch.distributed as dist

    import distspmm_b200 as d
    from distspmm_b200 import planner
    from distspmm_b200.dist import TorchComm, distributed_plan

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    A = d.gen_rmat(11, seed=3)
    lb, ub = planner.bounds(A, world, rank, partition)
    local = planner.partition(A, lb, ub)
    comm = TorchComm()
    mine, plan = distributed_plan(comm, local, n_rolls=4, task_dist=task_dist)
    from distspmm_b200.dist import fetch_view
    own = fetch_view(plan, mine, "rank")  # per-rank fetch lists: this rank's own tiling
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), remap=plan.remap, n_col=plan.n_col, offsets=plan.offsets,
             merged=plan.merged, demand=plan.demand, bounds=np.array([lb, ub]), own_n_col=own.n_col,
             own_merged=own.merged)
    assert comm.allreduce_max(float(rank)) == world - 1
    assert comm.allreduce_sum_i64(rank + 1) == world * (world + 1) // 2
    hs = comm.allgather_bytes(bytes([rank] * 64))
    assert [h[0] for h in hs] == list(range(world))
    comm.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,task_dist,partition", [(2, 2, "rows"), (3, 2, "rows"), (2, 0, "rows"),
                                                       (3, 2, "balanced")])
def test_distributed_plan_matches_in_process(world, task_dist, partition):
    import distspmm_b200 as d
    from distspmm_b200 import planner
    from distspmm_b200.dist import global_plan
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_worker, args=(world, _free_port(), tmp, task_dist, partition), nprocs=world,
                           start_method="spawn", join=True)
        A = d.gen_rmat(11, seed=3)
        T = world * 4
        bnd = [planner.bounds(A, world, p, partition) for p in range(world)]
        tl = [planner.tile(planner.partition(A, *b), T) for b in bnd]
        ref = global_plan(tl, task_dist, 4)
        for r in range(world):
            z = np.load(os.path.join(tmp, f"r{r}.npz"))
            assert tuple(z["bounds"]) == bnd[r]  # every rank derives the same row ranges
            assert np.array_equal(z["own_n_col"], tl[r].n_col) and np.array_equal(z["own_merged"], tl[r].needed)
            assert np.array_equal(z["remap"], ref.remap)
            assert np.array_equal(z["n_col"], ref.n_col)
            assert np.array_equal(z["offsets"], ref.offsets)
            assert np.array_equal(z["merged"], ref.merged)
            assert np.array_equal(z["demand"], ref.demand)


def _lonely(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from distspmm_b200.dist import TorchComm
    if rank == 1:
        return  # this rank never joins
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=3))
        TorchComm().allgather_i32(np.arange(4))
        res = "no error"
    except Exception as e:  # noqa: BLE001 - any timeout / store error is the expected outcome
        res = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(res)


def test_missing_rank_times_out_with_error():
    with tempfile.TemporaryDirectory() as tmp:
        mp.start_processes(_lonely, args=(2, _free_port(), tmp), nprocs=2, start_method="spawn", join=True)
        assert open(os.path.join(tmp, "r0.txt")).read().startswith("error")
