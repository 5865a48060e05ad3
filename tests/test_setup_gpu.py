"""The GPU set-up path: tiling, needed lists and the node union computed on the device
are identical to the host planner's (which is bit-exact with the oracle)."""
import numpy as np
import pytest

import distspmm_b200 as d
from distspmm_b200 import planner

pytestmark = pytest.mark.gpu


def _cols(local):
    import torch
    return torch.from_numpy(np.ascontiguousarray(local.indices, np.int64)).cuda()


@pytest.mark.parametrize("kind,kw", [("rmat", dict(scale=13)), ("stencil27", dict(n=16)),
                                     ("uniform", dict(rows=5000, nnz_per_row=7))])
@pytest.mark.parametrize("P,T", [(1, 1), (2, 8), (3, 7), (4, 32), (8, 32)])
def test_tile_device_matches_host(gpu, kind, kw, P, T):
    A = d.make_matrix(kind, seed=9, **kw)
    for p in range(P):
        lb, ub = planner.partition_bounds(A.num_rows, P, p)
        loc = planner.partition(A, lb, ub)
        h = planner.tile(loc, T)
        g = planner.tile_device(_cols(loc), A.num_cols, T)
        assert g.cpt == h.cpt
        for f in ("n_col", "n_slice", "nnz", "offsets", "needed"):
            assert np.array_equal(getattr(g, f), getattr(h, f)), f


@pytest.mark.parametrize("P,T", [(2, 8), (4, 16), (8, 32)])
def test_node_union_from_presence_max(gpu, P, T):
    """max of the ranks' presence maps -> the union lists of merge_needed."""
    import torch
    A = d.gen_rmat(12, seed=3)
    tilings, maps = [], []
    for p in range(P):
        loc = planner.partition(A, *planner.bounds(A, P, p, "balanced"))
        c = _cols(loc)
        tilings.append(planner.tile(loc, T))
        maps.append(planner.col_presence(c, A.num_cols))
    union = torch.stack(maps).max(dim=0).values.contiguous()
    n, off, cols = planner.needed_from_presence(union, A.num_cols, T)
    demand = np.stack([t.n_col for t in tilings]).astype(np.int32)
    n_ref, off_ref, cols_ref = planner.merge_needed(demand, np.concatenate([t.needed for t in tilings]))
    assert np.array_equal(n, n_ref) and np.array_equal(off, off_ref) and np.array_equal(cols, cols_ref)


def test_presence_rejects_out_of_range_columns(gpu):
    import torch
    bad = torch.tensor([0, 5, 10], dtype=torch.int64, device="cuda")
    with pytest.raises(d.DspError) as e:
        planner.col_presence(bad, 10)
    assert e.value.code == -3
    empty = torch.zeros(0, dtype=torch.int64, device="cuda")
    t = planner.tile_device(empty, 100, 4)
    assert t.n_col.sum() == 0 and t.nnz.sum() == 0 and t.needed.size == 0
