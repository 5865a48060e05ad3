"""dsp_spmm_csr_f32_noalloc — the SpMM entry point that allocates no device memory.

It serves callers that cannot call cudaMalloc (a latency-critical stream beside other work,
where cudaMalloc / cudaFree may synchronise the device; a framework whose own memory pool
owns the GPU; a step that must not fail with out-of-memory midway). Its scratch is a static
device array shared by every call on a device, so this test checks two calls in a row
through the C ABI: the second must not be disturbed by what the first left in the scratch.
Both results are compared with the plan-based entry point dsp_spmm_f32 and with the CPU
oracle (double accumulation), within the tolerance of the other parity tests,
|dC| <= 1e-5 * (|A|.|B|) elementwise. The cases cover the 128-bit and the scalar kernels
(N = 33), launches with several column blocks, and N = 2048 with 2^20 nonzeros, where the
chunk length grows so that two partial-row slots per chunk fit the static scratch.

This file is collected last (tests/test_zz_*) so that a run stopping at the first failure
has already run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import distspmm_b200 as d
import oracle

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def _noalloc(A, dA, B, C, accumulate):
    import torch
    from distspmm_b200 import _lib
    ip, ix, vv = dA
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("dsp_spmm_csr_f32_noalloc", ip.data_ptr(), ix.data_ptr(), vv.data_ptr(), A.num_rows, A.num_cols,
              A.nnz, B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0), B.shape[1], int(accumulate), stream)


def _matrices():
    n = 100_000  # one row far longer than a work chunk, between empty rows
    heavy = d.Csr(np.array([0, 0, n, n, n + 2], np.int64),
                  np.concatenate([np.arange(n), [3, 7]]).astype(np.int64),
                  np.random.default_rng(1).random(n + 2).astype(np.float32), 4, n)
    return [(d.gen_rmat(13, seed=2), 128), (d.gen_stencil27(20, seed=3), 64), (d.gen_uniform(3000, 9, seed=4), 100),
            (heavy, 32), (d.gen_rmat(12, seed=5), 33), (d.gen_uniform(1 << 15, 32, seed=6), 2048)]


@pytest.mark.parametrize("case", range(6))
def test_noalloc_two_calls_match_plan_entry_point(gpu, case):
    import torch
    from distspmm_b200.spmm import SpmmPlan
    A, N = _matrices()[case]
    dA = (torch.from_numpy(A.indptr).cuda(), torch.from_numpy(A.indices).cuda(), torch.from_numpy(A.values).cuda())
    B1 = d.dense_b(A.num_cols, N, seed=11)
    B2 = d.dense_b(A.num_cols, N, seed=12)
    plan = SpmmPlan(A, 0, N)
    ref1 = plan(torch.from_numpy(B1).cuda()).cpu().numpy().astype(np.float64)
    ref2 = plan(torch.from_numpy(B2).cuda()).cpu().numpy().astype(np.float64)
    exact1, abs1 = oracle.spmm_f64(A.indptr, A.indices, A.values, B1)
    exact2, abs2 = oracle.spmm_f64(A.indptr, A.indices, A.values, B2)

    C = torch.full((A.num_rows, N), float("nan"), device="cuda")  # every row must be written
    # call 1: C = A.B1
    _noalloc(A, dA, torch.from_numpy(B1).cuda(), C, accumulate=False)
    torch.cuda.synchronize()
    got1 = C.cpu().numpy()
    assert np.isfinite(got1).all()
    ok, worst = oracle.check_close(got1, ref1, abs1, RTOL)
    assert ok, f"first call vs dsp_spmm_f32: worst |dC| / tolerance = {worst:.3f}"
    ok, worst = oracle.check_close(got1, exact1, abs1, RTOL)
    assert ok, f"first call vs the oracle: worst |dC| / tolerance = {worst:.3f}"
    # call 2, right after, reusing the same static scratch: C += A.B2
    _noalloc(A, dA, torch.from_numpy(B2).cuda(), C, accumulate=True)
    torch.cuda.synchronize()
    got2 = C.cpu().numpy()
    ok, worst = oracle.check_close(got2, ref1 + ref2, abs1 + abs2, RTOL)
    assert ok, f"second call vs dsp_spmm_f32: worst |dC| / tolerance = {worst:.3f}"
    ok, worst = oracle.check_close(got2, exact1 + exact2, abs1 + abs2, RTOL)
    assert ok, f"second call vs the oracle: worst |dC| / tolerance = {worst:.3f}"


def test_noalloc_zero_size_call_sets_up_without_touching_memory(gpu):
    """A call with N = 0 or rows = 0 does the per-device set-up and writes nothing."""
    import torch
    from distspmm_b200 import _lib
    C = torch.full((4, 8), 7.0, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("dsp_spmm_csr_f32_noalloc", 0, 0, 0, 4, 4, 0, 0, 8, C.data_ptr(), 8, 0, 0, stream)
    _lib.call("dsp_spmm_csr_f32_noalloc", 0, 0, 0, 0, 4, 0, 0, 8, C.data_ptr(), 8, 8, 0, stream)
    torch.cuda.synchronize()
    assert bool((C == 7.0).all())


def test_noalloc_rejects_sizes_beyond_its_scratch(gpu):
    import torch
    from distspmm_b200 import _lib
    A = d.gen_uniform(64, 4, seed=1)
    ip, ix, vv = (torch.from_numpy(A.indptr).cuda(), torch.from_numpy(A.indices).cuda(),
                  torch.from_numpy(A.values).cuda())
    N = 2049  # DSP_NOALLOC_MAX_N + 1
    B = torch.zeros((A.num_cols, N), device="cuda")
    C = torch.zeros((A.num_rows, N), device="cuda")
    with pytest.raises(d.DspError) as e:
        _lib.call("dsp_spmm_csr_f32_noalloc", ip.data_ptr(), ix.data_ptr(), vv.data_ptr(), A.num_rows, A.num_cols,
                  A.nnz, B.data_ptr(), N, C.data_ptr(), N, N, 0, 0)
    assert e.value.code == -6 and "maximum" in str(e.value)
