"""dsp_comm_probe (the comm_test microbenchmark's measurement) on the GPU: the bulk copy
and the sparse gathers run and report device times; a peer GPU is used when there is one."""
import numpy as np
import pytest

from distspmm_b200 import comm_test

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("engine", ["lsu", "tma"])
@pytest.mark.parametrize("dims", [1, 4, 64, 128])
def test_probe_times(gpu, engine, dims):
    import torch
    peer = 1 if torch.cuda.device_count() > 1 else 0
    rows = 1 << 14
    perm = np.random.default_rng(0).permutation(rows).astype(np.int32)
    counts = [0, rows // 16, rows // 2, rows]
    bulk, sparse = comm_test.probe(0, peer, rows, dims, perm, counts, engine, reps=2)
    assert bulk > 0 and len(sparse) == 4
    assert all(t >= 0 for t in sparse) and sparse[3] > 0


def test_comm_test_cli_prints_reference_lines(gpu, capsys):
    assert comm_test.main(["20000", "4", "16", "2", "1", "10", "0"]) == 0
    lines = [ln for ln in capsys.readouterr().out.splitlines() if ln[:1].isdigit()]
    assert [ln.split(",")[0] for ln in lines] == ["4", "8", "16"]
    assert all(0.0 <= float(ln.split(",")[1]) <= 10 / 11 for ln in lines)
