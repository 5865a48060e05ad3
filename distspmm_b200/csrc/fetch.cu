// fetch.cu — sparsity-aware fetch of remote B rows over NVLink (the reference's
// comm_sparse_kernel / comm_sparse_aware, src/comm_man.h:72-101, which issues one
// nvshmemx_getmem_nbi_warp per needed row).
//
// dst[r, :] = src[r, :] for every global row r of a list, src being a peer GPU's B (CUDA IPC
// mapping or peer access) and dst this GPU's B, at the same row offsets.
//
// Two engines (dsp_rank_desc.fetch_engine):
//   LSU (default): 256-thread blocks, one per SM, each warp moving 4 rows at a time with
//     128-bit peer loads (32-bit for rows that are not float4 multiples). A block per SM
//     keeps ~2 MB in flight on NVLink (the link, not the SMs, bounds it) and leaves room on
//     every SM for the register-bound SpMM blocks that run at the same time.
//   TMA: each CTA is one warp with an 8-stage ring of shared-memory buffers; per stage it
//     issues one cp.async.bulk global->shared copy per row from the peer (completion
//     counted in bytes on the stage's mbarrier), then one cp.async.bulk shared->global copy
//     per row into local B. No multicast: every load reads the peer's memory once, into
//     this CTA's own shared memory. Per-row copies of 512 B carry enough per-request cost
//     that it needs about one CTA per SM to match the LSU engine on B200.
//     Every wait is bounded (about 2 s of clock64): on timeout the kernel sets *err, drains
//     its own copies (again bounded) and returns; dsp_rank_check_error() reports it.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "device.cuh"
#include "internal.h"
#include "mbar.cuh"

namespace dsp {

namespace {

constexpr int kStages = 8;
constexpr int kStageBytes = 16384;
constexpr long long kWaitCycles = kMbarWaitCycles;

// Self-test of the bounded wait: an mbarrier that nothing arrives at (a flag nothing sets).
__global__ void bounded_wait_selftest_kernel(long long budget, int *err) {
  __shared__ __align__(8) uint64_t mbar;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&mbar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  mbar_wait(smem_addr(&mbar), 0, err, 3, budget);
}

__global__ void __launch_bounds__(32) gather_rows_bulk_kernel(float *__restrict__ dst, const float *__restrict__ src,
                                                              const int32_t *__restrict__ rows, int64_t n,
                                                              int64_t ld, int row_bytes, int rows_per_stage,
                                                              int *err) {
  extern __shared__ __align__(128) unsigned char stage_buf[];
  __shared__ __align__(8) uint64_t mbar[kStages];
  const int lane = threadIdx.x;
  const int R = rows_per_stage;
  const int64_t G = gridDim.x, b = blockIdx.x;
  const int64_t groups = (n + R - 1) / R;
  const int64_t my = b < groups ? (groups - 1 - b) / G + 1 : 0;  // this CTA's groups b, b+G, ...
  if (my == 0) return;
  if (lane == 0) {
    for (int s = 0; s < kStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&mbar[s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();

  auto issue_loads = [&](int64_t i) {
    const int s = (int)(i % kStages);
    const int64_t r0 = (b + i * G) * R;
    const int cnt = (int)min((int64_t)R, n - r0);
    const uint32_t mb = smem_addr(&mbar[s]);
    if (lane == 0)
      asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(mb),
                   "r"(cnt * row_bytes)
                   : "memory");
    __syncwarp();
    for (int k = lane; k < cnt; k += 32) {
      const int64_t row = __ldg(rows + r0 + k);
      const uint32_t d = smem_addr(stage_buf + ((size_t)s * R + k) * row_bytes);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(d),
          "l"(src + row * ld), "r"(row_bytes), "r"(mb)
          : "memory");
    }
  };

  const int64_t prologue = min((int64_t)kStages, my);
  for (int64_t i = 0; i < prologue; ++i) issue_loads(i);
  int64_t consumed = 0;
  bool ok = true;
  for (int64_t i = 0; i < my; ++i) {
    const int s = (int)(i % kStages);
    if (!mbar_wait(smem_addr(&mbar[s]), (uint32_t)((i / kStages) & 1), err, 1)) {
      ok = false;
      break;
    }
    consumed = i + 1;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    const int64_t r0 = (b + i * G) * R;
    const int cnt = (int)min((int64_t)R, n - r0);
    for (int k = lane; k < cnt; k += 32) {
      const int64_t row = __ldg(rows + r0 + k);
      const uint32_t sp = smem_addr(stage_buf + ((size_t)s * R + k) * row_bytes);
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + row * ld), "r"(sp),
                   "r"(row_bytes)
                   : "memory");
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    // refill the stage of iteration i-1 once its stores have read it
    if (i >= 1 && i - 1 + kStages < my) {
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      __syncwarp();
      issue_loads(i - 1 + kStages);
    }
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  if (!ok) {
    // drain the loads still in flight (bounded) before the shared memory goes away
    const int64_t issued = min(my, max(prologue, consumed + kStages - 1));
    for (int64_t i = consumed; i < issued; ++i)
      if (!mbar_wait(smem_addr(&mbar[i % kStages]), (uint32_t)((i / kStages) & 1), err, 2)) break;
  }
}

__device__ __forceinline__ float4 ld_peer_v4(const float *p) {
  float4 v;
  asm volatile("ld.global.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

// One warp per group of kRows rows; all loads of the group are issued before the stores.
template <int kRows>
__global__ void __launch_bounds__(256) gather_rows_v4_kernel(float *__restrict__ dst, const float *__restrict__ src,
                                                             const int32_t *__restrict__ rows, int64_t n,
                                                             int64_t ld, int nvec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t g = warp * kRows; g < n; g += nwarps * kRows) {
    int32_t r[kRows];
#pragma unroll
    for (int k = 0; k < kRows; ++k) r[k] = g + k < n ? __ldg(rows + g + k) : -1;
    for (int v = lane; v < nvec; v += 32) {
      float4 x[kRows];
#pragma unroll
      for (int k = 0; k < kRows; ++k)
        if (r[k] >= 0) x[k] = ld_peer_v4(src + (int64_t)r[k] * ld + 4 * v);
#pragma unroll
      for (int k = 0; k < kRows; ++k)
        if (r[k] >= 0) *reinterpret_cast<float4 *>(dst + (int64_t)r[k] * ld + 4 * v) = x[k];
    }
  }
}

__global__ void __launch_bounds__(256) gather_rows_f1_kernel(float *__restrict__ dst, const float *__restrict__ src,
                                                             const int32_t *__restrict__ rows, int64_t n,
                                                             int64_t ld, int dims) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t g = warp; g < n; g += nwarps) {
    const int64_t r = __ldg(rows + g);
    for (int c = lane; c < dims; c += 32) dst[r * ld + c] = src[r * ld + c];
  }
}

std::mutex g_attr_mu;
bool g_attr_set[64] = {};

int64_t fetch_ctas() {
  static const int64_t v = [] {
    const char *e = getenv("DSP_FETCH_CTAS");
    return e ? std::max<int64_t>(1, atoll(e)) : (int64_t)148;  // one CTA per SM: NVLink-bound
  }();
  return v;
}

}  // namespace

int launch_gather_rows(float *dst, const float *src, const int32_t *rows, int64_t n, int dims, int engine, int *err,
                       cudaStream_t s) {
  if (n <= 0) return DSP_OK;
  const int row_bytes = dims * (int)sizeof(float);
  const bool aligned = ((uintptr_t)dst & 15) == 0 && ((uintptr_t)src & 15) == 0;
  static const int64_t lsu_blocks = [] {
    const char *e = getenv("DSP_FETCH_BLOCKS");
    return e ? std::max<int64_t>(1, atoll(e)) : (int64_t)148;
  }();
  static const int lsu_rows = [] {
    const char *e = getenv("DSP_FETCH_ROWS");
    return e && atoi(e) == 8 ? 8 : 4;
  }();
  if (engine == DSP_FETCH_TMA && aligned && row_bytes % 16 == 0 && row_bytes <= kStageBytes && err) {
    const int R = std::max(1, std::min(32, kStageBytes / row_bytes));
    const int smem = kStages * R * row_bytes;
    int dev = 0;
    cudaGetDevice(&dev);
    {
      std::lock_guard<std::mutex> lk(g_attr_mu);
      if (dev >= 0 && dev < 64 && !g_attr_set[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gather_rows_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kStages * kStageBytes);
        if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "gather smem attribute: %s", cudaGetErrorString(e));
        g_attr_set[dev] = true;
      }
    }
    const int64_t groups = (n + R - 1) / R;
    const int64_t ctas = std::min<int64_t>(groups, fetch_ctas());
    gather_rows_bulk_kernel<<<(unsigned)ctas, 32, smem, s>>>(dst, src, rows, n, dims, row_bytes, R, err);
  } else if (aligned && dims % 4 == 0) {
    // one 256-thread block per SM by default: enough rows in flight for NVLink, while the
    // SpMM blocks (register-bound) still fit beside it on every SM
    const int64_t blocks = std::min<int64_t>(((n + lsu_rows - 1) / lsu_rows + 7) / 8, lsu_blocks);
    if (lsu_rows == 8)
      gather_rows_v4_kernel<8><<<(unsigned)blocks, 256, 0, s>>>(dst, src, rows, n, dims, dims / 4);
    else
      gather_rows_v4_kernel<4><<<(unsigned)blocks, 256, 0, s>>>(dst, src, rows, n, dims, dims / 4);
  } else {
    const int64_t blocks = std::min<int64_t>((n + 7) / 8, 148 * 8);
    gather_rows_f1_kernel<<<(unsigned)blocks, 256, 0, s>>>(dst, src, rows, n, dims, dims);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "gather launch: %s", cudaGetErrorString(e));
}

}  // namespace dsp

extern "C" int dsp_selftest_bounded_wait(long long budget_cycles, int *code_out) {
  DSP_TRY_ARG(code_out && budget_cycles > 0 && budget_cycles <= dsp::kWaitCycles,
              "dsp_selftest_bounded_wait: budget %lld", budget_cycles);
  int *d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(int));
  if (e != cudaSuccess) return dsp::fail(DSP_ERR_CUDA, "selftest: %s", cudaGetErrorString(e));
  cudaMemset(d, 0, sizeof(int));
  dsp::bounded_wait_selftest_kernel<<<1, 32>>>(budget_cycles, d);
  e = cudaDeviceSynchronize();
  int v = -1;
  if (e == cudaSuccess) e = cudaMemcpy(&v, d, sizeof v, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return dsp::fail(DSP_ERR_CUDA, "selftest: %s", cudaGetErrorString(e));
  *code_out = v;
  return v != 0 ? dsp::fail(DSP_ERR_TIMEOUT, "bounded wait gave up as designed (code %d)", v) : DSP_OK;
}

// ------------------------------------------------------------------ bulk vs sparse fetch probe
//
// The reference's comm_test microbenchmark (src/comm_test.cu:83-147) on this engine's two
// fetch paths: one copy-engine copy of a peer's whole rows x dims buffer (the bulk tile
// fetch) against the sparse fetch of the first counts[i] rows of `row_ids` (the gather
// kernel of `engine`), both from peer_device's memory into device's, timed with CUDA events
// on one stream (mean of `reps` launches after one untimed launch).
extern "C" int dsp_comm_probe(int device, int peer_device, int64_t rows, int dims, const int32_t *row_ids,
                              int n_counts, const int64_t *counts, int engine, int reps, double *bulk_ms,
                              double *sparse_ms) {
  using namespace dsp;
  DSP_TRY_ARG(rows >= 1 && rows <= INT32_MAX && dims >= 1 && row_ids && n_counts >= 0 && (n_counts == 0 || counts) &&
                  reps >= 1 && bulk_ms && (n_counts == 0 || sparse_ms),
              "dsp_comm_probe: bad argument");
  int64_t max_n = 0;
  for (int i = 0; i < n_counts; ++i) {
    DSP_TRY_ARG(counts[i] >= 0 && counts[i] <= rows, "dsp_comm_probe: counts[%d] = %lld", i, (long long)counts[i]);
    max_n = std::max(max_n, counts[i]);
  }
  for (int64_t i = 0; i < max_n; ++i)
    DSP_TRY_ARG(row_ids[i] >= 0 && row_ids[i] < rows, "dsp_comm_probe: row_ids[%lld] = %d", (long long)i, row_ids[i]);
  int prev = 0;
  cudaGetDevice(&prev);
  const size_t bytes = sizeof(float) * (size_t)rows * (size_t)dims;
  float *src = nullptr, *dst = nullptr;
  int32_t *d_rows = nullptr;
  int *d_err = nullptr;
  cudaStream_t s = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  int rc = DSP_OK;
  cudaError_t e = cudaSetDevice(peer_device);
  if (e == cudaSuccess) e = cudaMalloc(&src, bytes);
  if (e == cudaSuccess) e = cudaMemset(src, 0, bytes);
  if (e == cudaSuccess) e = cudaSetDevice(device);
  if (e == cudaSuccess && peer_device != device) {
    e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();
      e = cudaSuccess;
    }
  }
  if (e == cudaSuccess) e = cudaMalloc(&dst, bytes);
  if (e == cudaSuccess) e = cudaMalloc(&d_rows, sizeof(int32_t) * (size_t)std::max<int64_t>(max_n, 1));
  if (e == cudaSuccess && max_n > 0)
    e = cudaMemcpy(d_rows, row_ids, sizeof(int32_t) * (size_t)max_n, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&d_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(d_err, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreate(&e0);
  if (e == cudaSuccess) e = cudaEventCreate(&e1);
  if (e != cudaSuccess) rc = fail(DSP_ERR_CUDA, "dsp_comm_probe set-up: %s", cudaGetErrorString(e));

  auto timed = [&](auto &&launch, double *out) -> int {
    int r = launch();
    if (r) return r;
    cudaEventRecord(e0, s);
    for (int k = 0; k < reps && r == DSP_OK; ++k) r = launch();
    cudaEventRecord(e1, s);
    cudaError_t ee = cudaEventSynchronize(e1);
    if (r) return r;
    if (ee != cudaSuccess) return fail(DSP_ERR_CUDA, "dsp_comm_probe: %s", cudaGetErrorString(ee));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    *out = (double)ms / reps;
    return DSP_OK;
  };
  if (rc == DSP_OK)
    rc = timed(
        [&]() -> int {
          cudaError_t ce = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s);
          return ce == cudaSuccess ? DSP_OK : fail(DSP_ERR_CUDA, "bulk copy: %s", cudaGetErrorString(ce));
        },
        bulk_ms);
  for (int i = 0; i < n_counts && rc == DSP_OK; ++i)
    rc = timed([&]() { return launch_gather_rows(dst, src, d_rows, counts[i], dims, engine, d_err, s); }, &sparse_ms[i]);
  if (rc == DSP_OK) {
    int flag = 0;
    cudaMemcpy(&flag, d_err, sizeof flag, cudaMemcpyDeviceToHost);
    if (flag) rc = fail(DSP_ERR_TIMEOUT, "dsp_comm_probe: a fetch wait gave up (code %d)", flag);
  }
  if (s) cudaStreamSynchronize(s);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  if (s) cudaStreamDestroy(s);
  if (d_err) cudaFree(d_err);
  if (d_rows) cudaFree(d_rows);
  if (dst) cudaFree(dst);
  if (src) {
    cudaSetDevice(peer_device);
    cudaFree(src);
  }
  cudaSetDevice(prev);
  return rc;
}
