"""Parity of the sm_100a SpMM kernels (through the C ABI) with the CPU oracle, for both
work decompositions (row-split and nnz-split) and the automatic choice.

Tolerance (fp32, from the engine's specification): elementwise
    |C_gpu - C_ref| <= 1e-5 * (|A|.|B|)
where C_ref is the double-accumulated CSR x dense product of the same fp32 inputs.
"""
import numpy as np
import pytest

import distspmm_b200 as d
import oracle

pytestmark = pytest.mark.gpu
RTOL = 1e-5
VARIANTS = ["rows", "nnz"]


def _run(A, N, seed=3, accumulate=False, C0=None, dims_hint=None, variant=None):
    import torch
    from distspmm_b200.spmm import SpmmPlan
    B = d.dense_b(A.num_cols, N, seed)
    plan = SpmmPlan(A, 0, dims_hint or N, variant)
    Bt = torch.from_numpy(B).cuda()
    Ct = torch.from_numpy(C0).cuda() if C0 is not None else None
    C = plan(Bt, Ct, accumulate=accumulate)
    torch.cuda.synchronize()
    return B, C.cpu().numpy(), plan


def _check(A, B, C, C0=None):
    ref, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    if C0 is not None:
        ref = ref + C0
        ab = ab + np.abs(C0)
    ok, worst = oracle.check_close(C, ref, ab, RTOL)
    assert np.isfinite(C).all()
    assert ok, f"worst |dC| / (1e-5 |A||B|) = {worst:.3f}"
    return worst


@pytest.fixture(scope="module")
def rmat13():
    return d.gen_rmat(13, seed=2)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("N", [1, 3, 4, 8, 16, 32, 64, 96, 100, 128, 256, 384, 512, 640])
def test_rmat_widths(gpu, rmat13, N, variant):
    B, C, plan = _run(rmat13, N, variant=variant)
    info = plan.info()
    assert info["variant"] == VARIANTS.index(variant)
    if variant == "rows":
        # pieces hold at most ~32K multiply-adds: the hub rows (max degree ~2.2K) are split
        # from N = 16 up
        assert (info["pieces"] > 0) == (info["max_row_len"] > info["piece_cap"])
        if N >= 16:
            assert info["pieces"] > 0
    else:
        assert info["items"] == -(-rmat13.nnz // info["piece_cap"])  # chunks of equal nonzeros
    _check(rmat13, B, C)


@pytest.mark.parametrize("variant", VARIANTS + [None])
@pytest.mark.parametrize("kind,kw,N", [
    ("rmat", dict(scale=15), 32),   # configuration 1 of the benchmark set
    ("stencil27", dict(n=24), 128),
    ("uniform", dict(rows=1 << 14, nnz_per_row=32), 256),
])
def test_matrix_families(gpu, kind, kw, N, variant):
    A = d.make_matrix(kind, seed=4, **kw)
    B, C, _ = _run(A, N, variant=variant)
    _check(A, B, C)


def test_variant_choice_follows_row_statistics(gpu):
    from distspmm_b200.spmm import SpmmPlan
    assert SpmmPlan(d.gen_rmat(12, seed=1), 0, 128).info()["variant"] == 1      # skewed, many empty rows
    assert SpmmPlan(d.gen_stencil27(12, seed=1), 0, 128).info()["variant"] == 0  # regular rows


@pytest.mark.parametrize("variant", VARIANTS)
def test_accumulate(gpu, rmat13, variant):
    C0 = d.dense_b(rmat13.num_rows, 128, seed=77)
    B, C, _ = _run(rmat13, 128, accumulate=True, C0=C0.copy(), variant=variant)
    _check(rmat13, B, C, C0)


@pytest.mark.parametrize("variant", VARIANTS)
def test_deterministic(gpu, rmat13, variant):
    _, C1, _ = _run(rmat13, 128, variant=variant)
    _, C2, _ = _run(rmat13, 128, variant=variant)
    assert np.array_equal(C1, C2)  # fixed summation order, no atomics


@pytest.mark.parametrize("variant", VARIANTS)
def test_strided_and_unaligned_operands(gpu, rmat13, variant):
    """B and C as column windows of wider buffers (ld > N, not 16-byte aligned: the
    scalar kernel path)."""
    import torch
    from distspmm_b200.spmm import SpmmPlan
    N = 64
    Bw = d.dense_b(rmat13.num_cols, N + 3, seed=5)
    plan = SpmmPlan(rmat13, 0, N, variant)
    Bt = torch.from_numpy(Bw).cuda()
    Cw = torch.full((rmat13.num_rows, N + 5), 7.0, device="cuda")
    plan(Bt[:, 1:N + 1], Cw[:, 2:N + 2])
    torch.cuda.synchronize()
    C = Cw.cpu().numpy()
    assert (C[:, :2] == 7).all() and (C[:, N + 2:] == 7).all()  # nothing written outside the window
    _check(rmat13, np.ascontiguousarray(Bw[:, 1:N + 1]), C[:, 2:N + 2])


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("N", [64, 128, 256, 512])
@pytest.mark.parametrize("pad,offset", [(4, 0), (8, 4), (0, 0)])
def test_vector_widths(gpu, rmat13, variant, N, pad, offset):
    """256-bit vectors need ld % 8 == 0 and 32-byte aligned rows; windows with ld % 8 == 4
    or a 16-byte offset take the float4 kernels instead. All three agree with the oracle."""
    import torch
    from distspmm_b200.spmm import SpmmPlan
    ld = N + pad
    Bw = d.dense_b(rmat13.num_cols, ld, seed=6)
    plan = SpmmPlan(rmat13, 0, N, variant)
    Bt = torch.from_numpy(Bw).cuda()
    Cw = torch.full((rmat13.num_rows, ld), 7.0, device="cuda")
    plan(Bt[:, offset:offset + N], Cw[:, offset:offset + N])
    torch.cuda.synchronize()
    C = Cw.cpu().numpy()
    assert (C[:, :offset] == 7).all() and (C[:, offset + N:] == 7).all()
    _check(rmat13, np.ascontiguousarray(Bw[:, offset:offset + N]), C[:, offset:offset + N])


@pytest.mark.parametrize("variant", VARIANTS)
def test_edge_cases(gpu, variant):
    import torch
    from distspmm_b200.spmm import SpmmPlan
    # all rows empty (C must still be written: poison it first)
    E = d.Csr(np.zeros(11, np.int64), np.zeros(0, np.int64), np.zeros(0, np.float32), 10, 10)
    plan = SpmmPlan(E, 0, 32, variant)
    C = torch.full((10, 32), float("nan"), device="cuda")
    plan(torch.ones((10, 32), device="cuda"), C)
    assert (C.cpu().numpy() == 0).all()
    # one huge row (forces many pieces / chunks) among empty rows, and a single-row matrix
    n = 200_000
    idx = np.arange(n, dtype=np.int64)
    H = d.Csr(np.array([0, 0, n, n], np.int64), idx, np.random.default_rng(1).random(n).astype(np.float32), 3, n)
    B, C, plan = _run(H, 128, variant=variant)
    assert plan.info()["pieces"] >= n // plan.info()["piece_cap"]
    _check(H, B, C)
    R = d.Csr(np.array([0, 3], np.int64), np.array([0, 1, 2], np.int64), np.ones(3, np.float32), 1, 3)
    B, C, _ = _run(R, 5, variant=variant)
    _check(R, B, C)
    # empty rows at both ends and between rows of a chunk; one nonzero per row
    G = d.Csr(np.array([0, 0, 0, 1, 1, 2, 3, 3, 3], np.int64), np.array([4, 0, 7], np.int64),
              np.array([2.0, 3.0, 5.0], np.float32), 8, 8)
    plan = SpmmPlan(G, 0, 16, variant)
    Bg = d.dense_b(8, 16, seed=1)
    C = torch.full((8, 16), float("nan"), device="cuda")
    plan(torch.from_numpy(Bg).cuda(), C)
    torch.cuda.synchronize()
    _check(G, Bg, C.cpu().numpy())
    # zero-width B
    plan = SpmmPlan(R, 0, 4, variant)
    plan(torch.zeros((3, 0), device="cuda"))


def test_nonaccumulating_launch_overwrites_every_row(gpu, rmat13):
    """C starts as NaN; every row, empty ones included, must be written."""
    import torch
    from distspmm_b200.spmm import SpmmPlan
    for variant in VARIANTS:
        plan = SpmmPlan(rmat13, 0, 128, variant)
        B = d.dense_b(rmat13.num_cols, 128, seed=3)
        C = torch.full((rmat13.num_rows, 128), float("nan"), device="cuda")
        plan(torch.from_numpy(B).cuda(), C)
        torch.cuda.synchronize()
        _check(rmat13, B, C.cpu().numpy())


def test_reference_run_mode_b_all_ones(gpu):
    """The reference runs with B = 1 (src/dist_spmm_node.cu:192): C[i,:] = row sum of A."""
    import torch
    from distspmm_b200.spmm import SpmmPlan
    A = d.gen_stencil27(16, seed=9)
    plan = SpmmPlan(A, 0, 128)
    C = plan(torch.ones((A.num_cols, 128), device="cuda")).cpu().numpy()
    rs = np.add.reduceat(A.values.astype(np.float64), A.indptr[:-1])
    assert np.allclose(C, rs[:, None], rtol=0, atol=1e-5 * 52)


@pytest.mark.parametrize("kind,kw,N", [("rmat", dict(scale=13), 128), ("stencil27", dict(n=20), 64),
                                       ("uniform", dict(rows=8192, nnz_per_row=24), 256)])
def test_agrees_with_cusparse(gpu, kind, kw, N):
    """The reference's arithmetic is cusparseSpMM (src/dist_spmm_node.cu:354-385); torch's
    sparse CSR product runs cuSPARSE on the same fp32 inputs. Both sit within the fp32
    tolerance of the exact product, so they agree within twice that (cuSPARSE is used here
    only as a checker)."""
    import torch
    A = d.make_matrix(kind, seed=12, **kw)
    B, C, _ = _run(A, N, seed=13)
    At = torch.sparse_csr_tensor(torch.from_numpy(A.indptr), torch.from_numpy(A.indices),
                                 torch.from_numpy(A.values), size=(A.num_rows, A.num_cols)).cuda()
    Cs = (At @ torch.from_numpy(B).cuda()).cpu().numpy()
    _, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, B)
    assert np.all(np.abs(C - Cs) <= 2 * RTOL * ab + 1e-30), float(np.max(np.abs(C - Cs) / (ab + 1e-30)))


def _banded(m, offsets, keep, seed):
    """m x m matrix with entries (i, i + o) for o in offsets where keep(i, o), values U(0.5, 1)."""
    rng = np.random.default_rng(seed)
    ip, ix = [0], []
    for i in range(m):
        cols = [i + o for o in offsets if 0 <= i + o < m and keep(i, o)]
        ix.extend(cols)
        ip.append(len(ix))
    vals = rng.uniform(0.5, 1.0, len(ix)).astype(np.float32)
    return d.Csr(np.array(ip, np.int64), np.array(ix, np.int64), vals, m, m)


# the diagonal kernel's configurations: TMA-staged windows (two CTA shapes) and the register
# kernel (8 or 4 rows per warp)
DIA_KERNELS = {
    "tma_7x2": {"DSP_SPMM_DIA_TMA": "1", "DSP_SPMM_DIA_TMA_SHAPE": "1"},
    "tma_15": {"DSP_SPMM_DIA_TMA": "1", "DSP_SPMM_DIA_TMA_SHAPE": "2"},
    "tma_6x2": {"DSP_SPMM_DIA_TMA": "1", "DSP_SPMM_DIA_TMA_SHAPE": "3"},
    "tma_3x3": {"DSP_SPMM_DIA_TMA": "1", "DSP_SPMM_DIA_TMA_SHAPE": "4"},
    "tma_7x2_wait_hint": {"DSP_SPMM_DIA_TMA": "1", "DSP_SPMM_DIA_TMA_SHAPE": "1", "DSP_SPMM_WAIT_HINT_NS": "2000"},
    "reg_8": {"DSP_SPMM_DIA_TMA": "0", "DSP_SPMM_DIA_ROWS": "8"},
    "reg_4": {"DSP_SPMM_DIA_TMA": "0", "DSP_SPMM_DIA_ROWS": "4"},
}


def _dia_kernel(monkeypatch, name):
    for k, v in DIA_KERNELS[name].items():
        monkeypatch.setenv(k, v)


@pytest.mark.parametrize("kernel", list(DIA_KERNELS))
def test_banded_diagonal_kernel_absent_entries_read_nothing(gpu, monkeypatch, kernel):
    """Banded operands run on the diagonal kernel (each configuration). An entry that does
    not exist must not read B: B rows that no entry uses hold NaN, and C must stay finite and
    match the oracle. Rows near the matrix edges (windows reaching outside B), rows without
    entries, and row counts that are not a multiple of the 8-row blocks are included."""
    import torch
    _dia_kernel(monkeypatch, kernel)
    from distspmm_b200.spmm import SpmmPlan
    m, N = 1003, 128
    # offsets -2..2 (one run) and +-100 (single diagonals); column 500 and 777 are never used
    A = _banded(m, [-100, -2, -1, 0, 1, 2, 100],
                lambda i, o: i + o not in (500, 777) and i % 97 != 13, seed=3)
    B = d.dense_b(m, N, 5)
    B[[500, 777]] = np.nan
    plan = SpmmPlan(A, 0, N)
    assert plan.info()["variant"] == 0  # banded: the diagonal kernel, though rows hold <= 7 entries
    C = plan(torch.from_numpy(B).cuda()).cpu().numpy()
    assert np.isfinite(C).all()
    Bz = B.copy()
    Bz[[500, 777]] = 0
    ref, ab = oracle.spmm_f64(A.indptr, A.indices, A.values, Bz)
    ok, worst = oracle.check_close(C, ref, ab, RTOL)
    assert ok, worst
    # accumulate: C += A.B
    C0 = d.dense_b(m, N, 9)
    C2 = plan(torch.from_numpy(B).cuda(), torch.from_numpy(C0.copy()).cuda(), accumulate=True).cpu().numpy()
    ok, worst = oracle.check_close(C2, ref + C0, ab + np.abs(C0), RTOL)
    assert ok, worst
    plan.check_error()


@pytest.mark.parametrize("kernel", list(DIA_KERNELS))
def test_banded_explicit_zero_still_reads_its_b_row(gpu, monkeypatch, kernel):
    """An explicit 0.0 in A is an entry: its B row is read, so a NaN there gives NaN in C,
    exactly as the CSR product (and the oracle) gives."""
    import torch
    _dia_kernel(monkeypatch, kernel)
    from distspmm_b200.spmm import SpmmPlan
    m, N = 64, 128
    A = _banded(m, [-1, 0, 1], lambda i, o: True, seed=4)
    row, col = 10, 11  # entry (10, 11)
    k = int(np.nonzero(A.indices[A.indptr[row]:A.indptr[row + 1]] == col)[0][0]) + int(A.indptr[row])
    A.values[k] = 0.0
    B = d.dense_b(m, N, 6)
    B[col] = np.nan
    C = SpmmPlan(A, 0, N)(torch.from_numpy(B).cuda()).cpu().numpy()
    nan_rows = sorted(set(np.nonzero(~np.isfinite(C))[0].tolist()))
    assert nan_rows == [10, 11, 12]  # every row with an entry in column 11, the zero included


@pytest.mark.parametrize("kernel", list(DIA_KERNELS))
def test_stencil_diagonal_kernel_widths(gpu, monkeypatch, kernel):
    """The 27-point stencil (the banded benchmark matrix) at several widths: N = 128 and 256
    use the diagonal kernel, N = 64 and 100 the row kernels; all match the oracle."""
    _dia_kernel(monkeypatch, kernel)
    A = d.gen_stencil27(14, seed=7)
    for N in (64, 100, 128, 256):
        B, C, plan = _run(A, N)
        _check(A, B, C)
        plan.check_error()


@pytest.mark.parametrize("kernel", ["tma_7x2", "tma_15", "tma_6x2", "tma_3x3", "tma_7x2_wait_hint"])
def test_banded_tma_windows_many_items_per_cta(gpu, monkeypatch, kernel):
    """Enough rows that every persistent CTA of the TMA-staged kernel takes many items, so
    its stage ring wraps many times (bounded waits on both barriers of every stage); holes
    in the band take the per-entry path. Results match the oracle and are bit-identical
    across runs."""
    import torch
    from distspmm_b200.spmm import SpmmPlan
    _dia_kernel(monkeypatch, kernel)
    m, N = 150_001, 256
    rng = np.random.default_rng(11)
    holes = rng.random((m, 7)) < 0.02
    offs = [-300, -2, -1, 0, 1, 2, 300]
    A = _banded(m, offs, lambda i, o: not holes[i, offs.index(o)], seed=12)
    B = d.dense_b(m, N, 13)
    plan = SpmmPlan(A, 0, N)
    assert plan.info()["variant"] == 0
    Bt = torch.from_numpy(B).cuda()
    C1 = plan(Bt)
    C2 = plan(Bt)
    torch.cuda.synchronize()
    plan.check_error()
    assert torch.equal(C1, C2)
    _check(A, B, C1.cpu().numpy())
