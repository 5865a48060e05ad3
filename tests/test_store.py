"""The host collectives of one-process-per-rank runs (dsp_store_*: the file-directory
rendezvous that replaces the reference's MPI Gather / Bcast / Allgather(v) / Allreduce on
one node), exercised by real processes on the CPU: values arrive complete and in rank
order, and a rank that never joins makes the others fail with DSP_ERR_TIMEOUT within the
bound instead of hanging."""
import ctypes
import multiprocessing as mp
import os

import numpy as np
import pytest

DSP_ERR_TIMEOUT = -7


def _member(rank, world, path, timeout_s, q):
    from distspmm_b200 import _lib
    L = _lib.lib()
    s = ctypes.c_void_p()
    try:
        _lib.call("dsp_store_open", path.encode(), rank, world, timeout_s, ctypes.byref(s))
        mine = np.arange(rank + 1, dtype=np.int32) + 100 * rank  # ragged: rank r sends r+1 ints
        sizes = (ctypes.c_int64 * world)()
        out = np.zeros(world * (world + 1) // 2, np.int32)
        rc = L.dsp_store_allgather(s, b"ragged", mine.ctypes.data, mine.nbytes, out.ctypes.data, out.nbytes, sizes)
        if rc != 0:
            q.put((rank, rc, None, None))
            L.dsp_store_close(s, 0)
            return
        rc = L.dsp_store_barrier(s, b"after")
        q.put((rank, rc, list(sizes), out.tolist()))
        L.dsp_store_close(s, 1 if rc == 0 else 0)
    except Exception as e:  # noqa: BLE001 — report to the parent
        q.put((rank, -99, str(e), None))


def _run(world, present, timeout_s, path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_member, args=(r, world, path, timeout_s, q)) for r in present]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(60)
    return sorted(res, key=lambda x: x[0])


def test_store_allgather_ragged_in_rank_order(tmp_path):
    world = 3
    path = str(tmp_path / "store")
    res = _run(world, range(world), 60.0, path)
    expect = [v for r in range(world) for v in (np.arange(r + 1) + 100 * r).tolist()]
    for rank, rc, sizes, out in res:
        assert rc == 0, (rank, rc, sizes)
        assert sizes == [4 * (r + 1) for r in range(world)]
        assert out == expect
    assert not os.path.exists(path)  # rank 0 removed the directory after every rank's last call


def test_store_rank_that_never_joins_times_out(tmp_path):
    res = _run(3, [0, 1], 1.0, str(tmp_path / "store"))  # rank 2 never starts
    assert [r[1] for r in res] == [DSP_ERR_TIMEOUT, DSP_ERR_TIMEOUT]


def test_store_rejects_bad_arguments(tmp_path):
    from distspmm_b200 import _lib
    import distspmm_b200 as d
    s = ctypes.c_void_p()
    with pytest.raises(d.DspError):
        _lib.call("dsp_store_open", str(tmp_path).encode(), 3, 2, 1.0, ctypes.byref(s))
    _lib.call("dsp_store_open", str(tmp_path / "s").encode(), 0, 1, 1.0, ctypes.byref(s))
    with pytest.raises(d.DspError):  # keys are file names: no directory separators
        _lib.call("dsp_store_allgather", s, b"a/b", None, 0, None, 0, None)
    _lib.call("dsp_store_barrier", s, b"ok")
    _lib.lib().dsp_store_close(s, 1)
