// run_rank.cpp — one rank of the dist_spmm_node program when every rank is its own process
// (`mpirun -np P dist_spmm_node ...`, srun, torchrun: src/dist_spmm_node.cu:20-25 and
// src/utils.h:176-237 bind each process to the GPU of its node-local rank).
//
// The stages and the report are those of dsp_run (src/dist_spmm_node.cu:61-437); the MPI
// collectives become dsp_store collectives in a directory shared by the job's processes:
//   demand rows n_col_list (Gather to the root + Bcast of the remap, src/utils.h:358-437):
//       all-gathered; every rank computes the same allocation;
//   needed sets (Allgather + Allgatherv, src/utils.h:439-547): all-gathered, merged;
//   B buffers: CUDA IPC handles all-gathered, each peer's B opened once;
//   per-rep times, traffic, memory (Allreduce MAX / SUM, src/dist_spmm_node.cu:401-409).
// A rank reads only its own rows of the matrix files (dsp_csr_load_rows) instead of the
// whole matrix as the reference's ranks do.
#include <cuda_runtime.h>
#include <string.h>

#include <chrono>

#include "internal.h"

using namespace dsp;

namespace {

double now_ms() {
  using namespace std::chrono;
  return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

struct Csr {
  dsp_csr m{};
  ~Csr() { dsp_csr_free(&m); }
};

struct Rank {
  dsp_rank *r = nullptr;
  ~Rank() { dsp_rank_destroy(r); }
};

int allgather_fixed(dsp_store *s, const char *key, const void *mine, int64_t bytes, int world, void *all) {
  return dsp_store_allgather(s, key, mine, bytes, all, bytes * world, nullptr);
}

}  // namespace

extern "C" int dsp_run_rank(const dsp_args *A, int me, int P, int device, dsp_store *store, dsp_report *rep) {
  DSP_TRY_ARG(A && rep && store, "dsp_run_rank: null argument");
  DSP_TRY_ARG(P >= 1 && me >= 0 && me < P, "dsp_run_rank: rank %d of %d", me, P);
  DSP_TRY_ARG(A->dims >= 1 && A->n_rolls >= 1 && A->repeat >= 0, "dsp_run_rank: dims %d n_rolls %d repeat %d",
              A->dims, A->n_rolls, A->repeat);
  DSP_TRY_ARG(A->task_dist >= 0 && A->task_dist <= 2, "Wrong task distribution type.");
  DSP_TRY_ARG(A->comm_type >= 0 && A->comm_type <= 2, "comm_type %d (expected 0, 1 or 2)", A->comm_type);
  DSP_TRY_ARG(A->file || A->matrix, "dsp_run_rank: no matrix");
  memset(rep, 0, sizeof *rep);
  const int dims = A->dims, T = A->n_rolls * P;
  DSP_TRY_ARG(T <= (int)(sizeof rep->remap / sizeof rep->remap[0]), "dsp_run_rank: %d tiles exceed the report", T);
  const char *part_env = getenv("DSP_PARTITION"), *scope_env = getenv("DSP_FETCH_SCOPE");
  const bool balanced = part_env && strcmp(part_env, "balanced") == 0;
  const bool per_rank = scope_env && strcmp(scope_env, "rank") == 0;
  const char *pipe_env = getenv("DSP_PIPELINE");
  const int pipeline = !pipe_env                        ? DSP_PIPELINE_AUTO
                       : strcmp(pipe_env, "rows") == 0  ? DSP_PIPELINE_ROWS
                       : strcmp(pipe_env, "split") == 0 ? DSP_PIPELINE_SPLIT
                       : strcmp(pipe_env, "groups") == 0 ? DSP_PIPELINE_GROUPS
                                                        : DSP_PIPELINE_AUTO;
  int rc;
  double t0;
  double stage[8] = {0};

  // 1 + 2. this rank's rows (src/dist_spmm_node.cu:61-99)
  t0 = now_ms();
  Csr local;
  int64_t M = 0, lb = 0, ub = 0, nnz_total = 0;  // nnz_total: summed over the ranks below
  if (A->file) {
    std::vector<int64_t> ip;
    if ((rc = dsp_csr_read_indptr(A->file, &M, nullptr))) return rc;
    if (balanced) {
      ip.resize((size_t)M + 1);
      if ((rc = dsp_csr_read_indptr(A->file, &M, ip.data()))) return rc;
      rc = dsp_partition_bounds_balanced(ip.data(), M, P, me, &lb, &ub);
    } else {
      rc = dsp_partition_bounds(M, P, me, &lb, &ub);
    }
    if (rc || (rc = dsp_csr_load_rows(A->file, lb, ub, &local.m))) return rc;
  } else {
    M = A->matrix->num_rows;
    rc = balanced ? dsp_partition_bounds_balanced(A->matrix->indptr, M, P, me, &lb, &ub)
                  : dsp_partition_bounds(M, P, me, &lb, &ub);
    if (rc || (rc = dsp_partition(A->matrix, lb, ub, &local.m))) return rc;
  }
  stage[0] = now_ms() - t0;
  {  // global nonzero count (for GFLOPS): sum over ranks
    int64_t all[4096];
    DSP_TRY_ARG(P <= 4096, "dsp_run_rank: %d ranks", P);
    if ((rc = allgather_fixed(store, "nnz", &local.m.nnz, 8, P, all))) return rc;
    nnz_total = 0;
    for (int p = 0; p < P; ++p) nnz_total += all[p];
  }
  rep->M = M;
  rep->nnz = nnz_total;
  rep->T = T;
  rep->row_lb = lb;
  rep->row_ub = ub;

  // 3. tiling and needed sets (src/dist_spmm_node.cu:102-132)
  t0 = now_ms();
  int64_t cpt = 0;
  std::vector<int32_t> my_ncol((size_t)T), my_nslice((size_t)T);
  std::vector<int64_t> my_off((size_t)T + 1);
  if ((rc = dsp_tile_counts(&local.m, T, &cpt, my_ncol.data(), my_nslice.data(), nullptr)) ||
      (rc = dsp_tile_needed(&local.m, T, my_off.data(), nullptr)))
    return rc;
  std::vector<int32_t> my_need((size_t)std::max<int64_t>(my_off[(size_t)T], 1));
  if ((rc = dsp_tile_needed(&local.m, T, my_off.data(), my_need.data()))) return rc;
  stage[2] = now_ms() - t0;

  // 4. allocation from every rank's demand row (src/dist_spmm_node.cu:134-168)
  t0 = now_ms();
  std::vector<int32_t> n_col((size_t)P * T);
  if ((rc = allgather_fixed(store, "ncol", my_ncol.data(), 4 * (int64_t)T, P, n_col.data()))) return rc;
  std::vector<int32_t> remap((size_t)T);
  if (A->task_dist == 0) {
    rc = dsp_alloc_slice(P, A->n_rolls, remap.data());
  } else if (A->task_dist == 1) {
    rc = dsp_alloc_random(P, A->n_rolls, 0x5eed, remap.data());
  } else {
    std::vector<int32_t> node((size_t)P, 0);  // one node
    const double h0 = now_ms();
    rc = dsp_hsdma(n_col.data(), P, T, node.data(), A->n_rolls, 5, 5, remap.data());
    rep->hsdma_ms = now_ms() - h0;
  }
  if (rc) return rc;
  memcpy(rep->remap, remap.data(), sizeof(int32_t) * (size_t)T);
  stage[3] = now_ms() - t0;

  // 5. node union of the needed sets (src/utils.h:439-547)
  t0 = now_ms();
  int64_t total_need = 0;
  for (int32_t c : n_col) total_need += c;
  std::vector<int32_t> flat((size_t)std::max<int64_t>(total_need, 1));
  if ((rc = dsp_store_allgather(store, "need", my_need.data(), 4 * my_off[(size_t)T], flat.data(), 4 * total_need,
                                nullptr)))
    return rc;
  std::vector<int64_t> moff((size_t)T + 1);
  std::vector<int32_t> mcount((size_t)T);
  if ((rc = dsp_merge_needed(P, T, n_col.data(), flat.data(), moff.data(), nullptr, mcount.data()))) return rc;
  std::vector<int32_t> merged((size_t)std::max<int64_t>(moff[(size_t)T], 1));
  if ((rc = dsp_merge_needed(P, T, n_col.data(), flat.data(), moff.data(), merged.data(), mcount.data()))) return rc;
  stage[4] = now_ms() - t0;

  // 6 + 7. device set-up and selector (src/dist_spmm_node.cu:184-251, src/comm_man.h:341-410)
  t0 = now_ms();
  dsp_comm_model intra, inter;
  if ((rc = dsp_comm_model_preset(A->platform, DSP_TIER_INTRA, &intra)) ||
      (rc = dsp_comm_model_preset(A->platform, DSP_TIER_INTER, &inter)))
    return rc;
  std::vector<uint8_t> sparse((size_t)T);
  const int32_t *counts = per_rank ? my_ncol.data() : mcount.data();
  const double s0 = now_ms();
  if ((rc = dsp_comm_select(A->comm_type, dims, &intra, &inter, T, counts, my_nslice.data(), sparse.data(), nullptr)))
    return rc;
  stage[6] = now_ms() - s0;
  dsp_rank_desc d{};
  d.rank = me;
  d.world = P;
  d.device = device;
  d.dims = dims;
  d.T = T;
  d.n_streams = A->n_streams > 0 ? A->n_streams : 4;
  d.cpt = cpt;
  d.M = M;
  d.m_lb = lb;
  d.local = &local.m;
  d.remap = remap.data();
  d.sparse = sparse.data();
  d.needed_offsets = per_rank ? my_off.data() : moff.data();
  d.needed_cols = per_rank ? my_need.data() : merged.data();
  d.n_slice = my_nslice.data();
  d.pipeline = pipeline;
  Rank R;
  if ((rc = dsp_rank_create(&d, &R.r))) return rc;
  if (cudaSetDevice(device) != cudaSuccess) return fail(DSP_ERR_CUDA, "cudaSetDevice(%d)", device);
  if (A->b_ones) {
    float *B = nullptr;
    dsp_rank_b_ptr(R.r, &B);
    std::vector<float> ones((size_t)std::min<int64_t>(M * dims, 1 << 24), 1.0f);
    for (int64_t o = 0; o < M * dims; o += (int64_t)ones.size()) {
      const size_t n = (size_t)std::min<int64_t>((int64_t)ones.size(), M * dims - o);
      if (cudaMemcpy(B + o, ones.data(), n * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(DSP_ERR_CUDA, "fill ones failed");
    }
  } else if ((rc = dsp_rank_fill_b(R.r, A->b_seed, nullptr))) {
    return rc;
  }
  // peers' B by CUDA IPC
  std::vector<char> handles((size_t)64 * P);
  char mine[64];
  if ((rc = dsp_rank_ipc_handle(R.r, mine)) ||
      (rc = allgather_fixed(store, "ipc", mine, 64, P, handles.data())))
    return rc;
  for (int q = 0; q < P; ++q)
    if (q != me && (rc = dsp_rank_open_peer(R.r, q, &handles[(size_t)64 * q]))) return rc;
  stage[5] = now_ms() - t0 - stage[6];

  // 8. streams
  t0 = now_ms();
  cudaStream_t stream = nullptr;
  if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess)
    return fail(DSP_ERR_CUDA, "stream create failed");
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } sg{stream};
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(DSP_ERR_CUDA, "set-up: %s", cudaGetErrorString(cudaGetLastError()));
  stage[7] = now_ms() - t0;
  // every rank's owned tiles hold B before any peer reads them
  if ((rc = dsp_store_barrier(store, "ready"))) return rc;

  // hot loop (src/dist_spmm_node.cu:329-394). B does not change between reps (peers read
  // only owned tiles, a rank writes only the rows it does not own), so the reps of
  // different ranks need no barrier between them; each rep is timed on its own rank.
  std::vector<double> reps((size_t)std::max(A->repeat, 1), 0.0);
  for (int it = 0; it < A->repeat; ++it) {
    const double s = now_ms();
    if ((rc = dsp_rank_step(R.r, stream))) return rc;
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "step: %s", cudaGetErrorString(e));
    reps[(size_t)it] = now_ms() - s;
  }
  if ((rc = dsp_rank_check_error(R.r))) return rc;
  // no peer reads this rank's B after this point
  if ((rc = dsp_store_barrier(store, "done"))) return rc;

  // statistics: per-rep and per-stage times MAX over ranks, traffic SUM, memory MAX
  int64_t traffic = 0;
  dsp_traffic_intra(me, T, remap.data(), sparse.data(), counts, my_nslice.data(), dims, &traffic);
  dsp_rank_stats st;
  dsp_rank_stats_get(R.r, &st);
  const int nr = (int)reps.size();
  std::vector<double> mine_stats((size_t)nr + 8 + 3);
  std::copy(reps.begin(), reps.end(), mine_stats.begin());
  std::copy(stage, stage + 8, mine_stats.begin() + nr);
  mine_stats[(size_t)nr + 8] = (double)traffic;
  mine_stats[(size_t)nr + 9] = (double)st.fetch_bytes;
  mine_stats[(size_t)nr + 10] = (double)st.device_bytes;
  std::vector<double> all(mine_stats.size() * (size_t)P);
  if ((rc = allgather_fixed(store, "stats", mine_stats.data(), 8 * (int64_t)mine_stats.size(), P, all.data())))
    return rc;
  std::vector<double> rep_max((size_t)nr, 0.0);
  for (int p = 0; p < P; ++p) {
    const double *x = &all[(size_t)p * mine_stats.size()];
    for (int i = 0; i < nr; ++i) rep_max[(size_t)i] = std::max(rep_max[(size_t)i], x[i]);
    for (int i = 0; i < 8; ++i) rep->stage_ms[i] = std::max(rep->stage_ms[i], x[nr + i]);
    rep->traffic_intra += (int64_t)x[nr + 8];
    rep->fetched_bytes += (int64_t)x[nr + 9];
    rep->mem_gb = std::max(rep->mem_gb, x[nr + 10] / (1024.0 * 1024.0 * 1024.0));
  }
  rep_max.resize((size_t)A->repeat);
  // the reference drops the first 5 reps (src/dist_spmm_node.cu:414-435); with fewer, all
  // of them count
  std::vector<double> kept(rep_max.size() > 5 ? rep_max.begin() + 5 : rep_max.begin(), rep_max.end());
  rep->reps_counted = (int)kept.size();
  if (!kept.empty()) {
    double sum = 0;
    for (double x : kept) sum += x;
    rep->avg_ms = sum / (double)kept.size();
    std::vector<double> s = kept;
    std::sort(s.begin(), s.end());
    rep->min_ms = s.front();
    rep->median_ms = s[s.size() / 2];
    rep->gflops = dsp_gflops(nnz_total, dims, rep->avg_ms);
  }
  if (A->c_out && ub > lb) {
    if ((rc = dsp_rank_download_c(R.r, A->c_out, stream))) return rc;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return fail(DSP_ERR_CUDA, "download C failed");
  }
  return DSP_OK;
}
