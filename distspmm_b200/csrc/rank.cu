// rank.cu — one GPU's share of the distributed SpMM.
//
// Data layout in HBM (per rank):
//   B     [M x dims] fp32 row-major, full height. The tiles this rank owns live at their
//         global row offsets; remote rows fetched for a step land at the same offsets, so
//         the SpMM kernels use global column ids unchanged and no receive buffer is ever
//         recycled (the reference's 4-slot ring of src/dist_spmm_node.cu:199-203 with its
//         reuse race, replaced by one full-height buffer: 180 GB HBM holds B at every
//         configuration this engine targets).
//   C     [m_local x dims] fp32 row-major.
//   A     one DevOperand per phase. Peers are visited in the reference's ring order
//         (me + k) % P (src/dist_spmm_node.cu:339-343). Rows pipeline: a local row belongs
//         to phase k, the latest ring position among the owners of its columns, and phase
//         k holds whole rows (all their nonzeros): every C row is written exactly once.
//         Phase 0 = rows that need only tiles this rank owns. Split pipeline: phase k holds
//         the nonzeros of ring position k; a row is written by its first phase and
//         accumulated by later ones (first_phase[] on the device).
//         Rows without nonzeros are listed apart and zero-filled.
//   scratch: partial rows of rows cut between work units, shared by the phases (they run
//         in order on one stream).
//
// One step: the fetch streams (high priority) pull each peer's tiles — bulk tiles with one
// copy-engine copy each (cudaMemcpyAsync over NVLink, as nvshmemx_getmem_on_stream in
// src/comm_man.h:503), sparse tiles with one gather kernel per peer that moves the merged
// needed rows with 128-bit loads from the peer's B (src/comm_man.h:72-101) — while the
// compute stream runs phase 0, then phase k as soon as the fetches of ring positions 1..k
// have landed. The reference instead accumulates every tile into C (beta = 1,
// src/dist_spmm_node.cu:371-383): one read-modify-write of C per tile, which phases avoid.
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include "device.cuh"
#include "internal.h"

namespace dsp {

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

#define DSP_CUDA(call)                                                                      \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(DSP_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

}  // namespace
}  // namespace dsp

using namespace dsp;

struct dsp_rank {
  int me = 0, P = 1, device = 0, dims = 0, T = 0, n_streams = 1, fetch_engine = DSP_FETCH_LSU;
  int *d_err = nullptr;  // set by a fetch or SpMM kernel whose bounded wait gave up
  int64_t cpt = 0, M = 0, m_lb = 0, m_local = 0, nnz_local = 0;
  float model_ms[3] = {0.f, 0.f, 0.f};  // modelled step of the rows / split / groups pipelines
  std::vector<int32_t> remap;
  std::vector<uint8_t> sparse;
  float *B = nullptr, *C = nullptr, *scratch = nullptr;
  int64_t scratch_floats = 0;

  struct Segment {
    int owner = 0;  // (me + k) % P
    DevOperand op;  // the rows of phase k
  };
  std::vector<Segment> segs;  // one per phase / ring position k
  int pipeline = DSP_PIPELINE_ROWS;
  uint8_t *d_first_phase = nullptr;  // split pipeline: first phase writing each local row
  int32_t *d_empty = nullptr;  // local rows without nonzeros (zero-filled each step)
  int64_t n_empty = 0;

  struct Fetch {
    std::vector<std::pair<int64_t, int64_t>> bulk;  // (first row, rows)
    int32_t *d_rows = nullptr;                      // sparse gather rows (global ids)
    int64_t n_rows = 0;
  };
  std::vector<Fetch> fetch;  // by segment index k (k = 0 unused)
  // groups pipeline: segs[g] holds row group g; gfetch[g * P + k] the rows of peer (me+k)%P
  // that group g is the first to need; bulk tiles (fetch[k].bulk) land before group 0
  int n_groups = 0;
  std::vector<int64_t> group_end;  // first local row after group g
  std::vector<Fetch> gfetch;
  std::vector<cudaEvent_t> ev_group;  // [g * P + k]

  std::vector<const float *> peer_B;
  std::vector<int> peer_dev;
  std::vector<bool> peer_ipc;
  std::vector<int64_t> owned;  // owned tiles

  cudaStream_t compute = nullptr;
  cudaStream_t side = nullptr;  // zero fill of the empty rows, beside the phases
  std::vector<cudaStream_t> fstreams;
  cudaEvent_t ev_start = nullptr, ev_c0 = nullptr, ev_c1 = nullptr, ev_zero = nullptr;
  std::vector<cudaEvent_t> ev_fetch, ev_fetch_begin, ev_seg_begin, ev_seg_end;  // per peer / segment
  std::vector<bool> fetch_ran, seg_ran;                                         // last step
  dsp_rank_stats stats{};
};

namespace {

// Split pipeline: phase k holds the nonzeros whose column tile is owned by ring position
// k (rows listed in ascending order, their nonzeros in column order); first[i] is the
// first phase touching row i, where the row is written, later phases adding to it.
int build_split_phases(dsp_rank *r, const dsp_csr *a, const std::vector<int32_t> &first) {
  const int P = r->P, me = r->me;
  const int64_t m = a->num_rows, nnz = a->nnz, cpt = r->cpt;
  std::vector<uint8_t> pos((size_t)std::max<int64_t>(nnz, 1));
  parallel_for(nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j) pos[(size_t)j] = (uint8_t)((r->remap[(size_t)(a->indices[j] / cpt)] - me + P) % P);
  }, 1 << 16);
  std::vector<uint8_t> fp((size_t)std::max<int64_t>(m, 1), 0xff);
  for (int64_t i = 0; i < m; ++i)
    if (first[(size_t)i] >= 0) fp[(size_t)i] = (uint8_t)first[(size_t)i];
  int rc = dev_upload(&r->d_first_phase, fp.data(), fp.size());
  if (rc) return rc;
  for (int k = 0; k < P; ++k) {
    auto &S = r->segs[(size_t)k];
    S.owner = (me + k) % P;
    std::vector<int32_t> rows;
    std::vector<int64_t> ptr(1, 0), idx;
    std::vector<float> val;
    for (int64_t i = 0; i < m; ++i) {
      const int64_t before = (int64_t)idx.size();
      for (int64_t j = a->indptr[i]; j < a->indptr[i + 1]; ++j)
        if (pos[(size_t)j] == k) {
          idx.push_back(a->indices[j]);
          val.push_back(a->values[j]);
        }
      if ((int64_t)idx.size() > before) {
        rows.push_back((int32_t)i);
        ptr.push_back((int64_t)idx.size());
      }
    }
    if (idx.empty()) {
      idx.push_back(0);
      val.push_back(0.f);
    }
    rc = S.op.upload(r->device, m, r->M, ptr.data(), rows.data(), (int64_t)rows.size(), idx.data(), val.data(), 0,
                     ptr.back(), r->dims, false);
    if (rc) return rc;
    r->scratch_floats = std::max(r->scratch_floats, S.op.pieces * (int64_t)r->dims);
  }
  return DSP_OK;
}

// Phase of every local row: the latest ring position (owner - me mod P) among its
// columns' tiles; -1 for rows without nonzeros. Phase k holds whole rows, so each row is
// computed once, with all its nonzeros, after the fetches of ring positions 1..k. The
// split pipeline (chosen here for DSP_PIPELINE_AUTO when less than half of the nonzeros
// would run before any fetch lands) cuts rows by ring position instead.
int build_groups(dsp_rank *r, const dsp_csr *a, int groups);

// Rows this rank's fetch moves per step (what build_fetch / build_group_fetch will list):
// whole bulk tiles and the sparse tiles' lists, for remote tiles holding local nonzeros.
int64_t planned_fetch_rows(const dsp_rank *r, const dsp_rank_desc *d) {
  if (r->P == 1) return 0;
  std::vector<int64_t> nnz_t((size_t)r->T, 0);
  for (int64_t j = 0; j < d->local->nnz; ++j) nnz_t[(size_t)(d->local->indices[j] / r->cpt)]++;
  int64_t rows = 0;
  for (int t = 0; t < r->T; ++t) {
    if (r->remap[(size_t)t] == r->me || nnz_t[(size_t)t] == 0) continue;
    rows += r->sparse[(size_t)t] ? d->needed_offsets[t + 1] - d->needed_offsets[t]
                                 : std::min<int64_t>(r->cpt, r->M - (int64_t)t * r->cpt);
  }
  return rows;
}

// Step-time model of the three phase structures for DSP_PIPELINE_AUTO, in seconds. One
// nonzero costs a B-row gather (dims x 4 bytes at ~10 TB/s through L2); one fetched row
// dims x 4 bytes over NVLink at ~730 GB/s; an accumulated piece a C-row read and write (two
// gathers' worth); every extra segment of the groups pipeline ~60 us (the partial last wave
// of its launch). Fitted to R-MAT 24 on 2 x B200 (per rank: split 13.95 / groups 14.42 /
// rows 16.00 ms on the hub rank, rows 14.30 / split 14.67 / groups 15.54 on the other).
struct PipelineModel {
  double rows, split, groups;
};

PipelineModel pipeline_model(int dims, int64_t nnz, int64_t phase0_nnz, int64_t local_nnz, int64_t split_pieces,
                             int64_t group_pieces, int64_t fetch_rows, int G) {
  const double t_nnz = dims * 4.0 / 10e12, t_fetch = fetch_rows * (dims * 4.0) / 730e9;
  const double all = nnz * t_nnz, p0 = phase0_nnz * t_nnz, loc = local_nnz * t_nnz;
  PipelineModel m;
  m.rows = std::max(t_fetch, p0) + (all - p0);
  m.split = std::max(t_fetch, loc) + (all - loc) + 2.0 * split_pieces * t_nnz;
  m.groups = std::max(t_fetch + (all - loc) / std::max(G, 1), all) + 2.0 * group_pieces * t_nnz + G * 60e-6;
  return m;
}

int build_phases(dsp_rank *r, const dsp_csr *a, int pipeline, int groups, int64_t fetch_rows) {
  const int P = r->P, me = r->me;
  const int64_t m = a->num_rows, cpt = r->cpt;
  std::vector<int32_t> phase((size_t)std::max<int64_t>(m, 1), -1), first((size_t)std::max<int64_t>(m, 1), -1);
  std::vector<uint8_t> touched((size_t)std::max<int64_t>(m, 1), 0);  // ring positions per row (P <= 64)
  parallel_for(m, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) {
      int32_t ph = -1, lo = P;
      uint64_t seen = 0;
      for (int64_t j = a->indptr[i]; j < a->indptr[i + 1]; ++j) {
        const int32_t k = (r->remap[(size_t)(a->indices[j] / cpt)] - me + P) % P;
        ph = std::max(ph, k);
        lo = std::min(lo, k);
        if (k < 64) seen |= 1ull << k;
      }
      phase[(size_t)i] = ph;
      first[(size_t)i] = ph < 0 ? -1 : lo;
      touched[(size_t)i] = (uint8_t)__builtin_popcountll(seen);
    }
  }, 1024);
  std::vector<int32_t> empty;
  int64_t rows_phase0_nnz = 0;
  for (int64_t i = 0; i < m; ++i) {
    if (phase[(size_t)i] < 0) empty.push_back((int32_t)i);
    if (phase[(size_t)i] == 0) rows_phase0_nnz += a->indptr[i + 1] - a->indptr[i];
  }
  r->n_empty = (int64_t)empty.size();
  if (r->n_empty) {
    int rc = dev_upload(&r->d_empty, empty.data(), sizeof(int32_t) * empty.size());
    if (rc) return rc;
  }
  r->segs.resize((size_t)P);
  // local_nnz: nonzeros in tiles this rank owns (what split and groups compute before any
  // fetch); acc_pieces: pieces (row, ring position) after each row's first one, which the split
  // pipeline accumulates into C; group_pieces: rows with both owned and remote nonzeros,
  // which the groups pipeline accumulates once
  int64_t local_nnz = 0, acc_pieces = 0, group_pieces = 0;
  for (int64_t i = 0; i < m; ++i) {
    if (touched[(size_t)i] > 1) acc_pieces += touched[(size_t)i] - 1;
    if (touched[(size_t)i] > 1 && first[(size_t)i] == 0) group_pieces++;
    for (int64_t j = a->indptr[i]; j < a->indptr[i + 1]; ++j)
      local_nnz += (r->remap[(size_t)(a->indices[j] / cpt)] - me + P) % P == 0;
  }
  // AUTO: whole rows when the rows needing only owned tiles hold at least half the
  // nonzeros (they hide the fetch: stencils); otherwise the structure with the shortest
  // modelled step, whole rows kept unless another is >= 3 % shorter (the model leaves out
  // the fetch kernels' share of the SMs, which weighs on the overlapped forms).
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>({groups > 0 ? groups : 8, std::max<int64_t>(m, 1), 253}));
  const PipelineModel model =
      pipeline_model(r->dims, a->nnz, rows_phase0_nnz, local_nnz, acc_pieces, group_pieces, fetch_rows, G);
  r->model_ms[0] = (float)(model.rows * 1e3);
  r->model_ms[1] = (float)(model.split * 1e3);
  r->model_ms[2] = (float)(model.groups * 1e3);
  if (pipeline == DSP_PIPELINE_AUTO) {
    pipeline = DSP_PIPELINE_ROWS;
    if (2 * rows_phase0_nnz < a->nnz) {
      const double best = std::min(model.split, model.groups);
      if (best < 0.97 * model.rows) pipeline = model.split <= model.groups ? DSP_PIPELINE_SPLIT : DSP_PIPELINE_GROUPS;
    }
  }
  if (P == 1 || P > 64) pipeline = DSP_PIPELINE_ROWS;
  r->pipeline = pipeline;
  if (pipeline == DSP_PIPELINE_GROUPS) return build_groups(r, a, groups);
  if (pipeline == DSP_PIPELINE_SPLIT) {
    r->stats.phase0_nnz = local_nnz;
    return build_split_phases(r, a, first);
  }
  r->stats.phase0_nnz = rows_phase0_nnz;
  for (int k = 0; k < P; ++k) {
    auto &S = r->segs[(size_t)k];
    S.owner = (me + k) % P;
    std::vector<int32_t> rows;
    std::vector<int64_t> src;  // first nonzero of each listed row in the local CSR
    std::vector<int64_t> ptr(1, 0);
    for (int64_t i = 0; i < m; ++i) {
      if (phase[(size_t)i] != k) continue;
      rows.push_back((int32_t)i);
      src.push_back(a->indptr[i]);
      ptr.push_back(ptr.back() + (a->indptr[i + 1] - a->indptr[i]));
    }
    const int64_t nr = (int64_t)rows.size(), nz = ptr.back();
    std::vector<int64_t> idx((size_t)std::max<int64_t>(nz, 1));
    std::vector<float> val((size_t)std::max<int64_t>(nz, 1));
    parallel_for(nr, [&](int64_t b, int64_t e) {
      for (int64_t q = b; q < e; ++q) {
        const int64_t n = ptr[(size_t)q + 1] - ptr[(size_t)q];
        memcpy(&idx[(size_t)ptr[(size_t)q]], a->indices + src[(size_t)q], sizeof(int64_t) * (size_t)n);
        memcpy(&val[(size_t)ptr[(size_t)q]], a->values + src[(size_t)q], sizeof(float) * (size_t)n);
      }
    }, 1024);
    // non-accumulating, but only the listed rows: no zero fill of the rows in between
    int rc = S.op.upload(r->device, m, r->M, ptr.data(), rows.data(), nr, idx.data(), val.data(), 0, nz, r->dims,
                         false);
    if (rc) return rc;
    r->scratch_floats = std::max(r->scratch_floats, S.op.pieces * (int64_t)r->dims);
  }
  return DSP_OK;
}

int build_fetch(dsp_rank *r, const dsp_rank_desc *d) {
  const int P = r->P, T = r->T;
  std::vector<int64_t> nnz_t((size_t)T, 0);
  for (int64_t j = 0; j < d->local->nnz; ++j) nnz_t[(size_t)(d->local->indices[j] / r->cpt)]++;
  r->fetch.assign((size_t)P, dsp_rank::Fetch());
  for (int k = 1; k < P; ++k) {
    const int q = (r->me + k) % P;
    auto &F = r->fetch[(size_t)k];
    std::vector<int32_t> rows;
    for (int t = 0; t < T; ++t) {  // tiles of q in ascending order (task_assignments[q])
      if (r->remap[(size_t)t] != q || nnz_t[(size_t)t] == 0) continue;  // src/dist_spmm_node.cu:344
      const int64_t row0 = (int64_t)t * r->cpt;
      if (r->sparse[(size_t)t]) {
        for (int64_t p = d->needed_offsets[t]; p < d->needed_offsets[t + 1]; ++p)
          rows.push_back((int32_t)(row0 + d->needed_cols[p]));
        r->stats.fetch_sparse_tiles++;
      } else {
        const int64_t n = std::min<int64_t>(r->cpt, r->M - row0);
        if (n > 0) F.bulk.push_back({row0, n});
        r->stats.fetch_bulk_tiles++;
        r->stats.fetch_rows += n;
      }
    }
    F.n_rows = (int64_t)rows.size();
    r->stats.fetch_rows += F.n_rows;
    if (F.n_rows) {
      int rc = dev_upload(&F.d_rows, rows.data(), sizeof(int32_t) * rows.size());
      if (rc) return rc;
    }
  }
  r->stats.fetch_bytes = r->stats.fetch_rows * (int64_t)r->dims * 4;
  return DSP_OK;
}

// Groups pipeline. Segment 0 holds the nonzeros of every row whose column tiles this rank
// owns (no fetch needed: it runs while group 0's rows arrive) and writes those rows; the
// local rows are cut into G contiguous groups of equal cost (nonzeros + rows), and segment
// g + 1 holds group g's remote nonzeros, adding to rows segment 0 wrote (first_phase) and
// writing the others. Every row is thus written once and read back at most once.
int build_groups(dsp_rank *r, const dsp_csr *a, int groups) {
  const int64_t m = a->num_rows;
  // at most 253 groups: segment numbers (first_phase) are bytes, 255 meaning "no nonzeros"
  const int G = (int)std::max<int64_t>(1, std::min<int64_t>({groups > 0 ? groups : 8, std::max<int64_t>(m, 1), 253}));
  const int me = r->me;
  r->n_groups = G;
  r->segs.assign((size_t)G + 1, dsp_rank::Segment());
  r->group_end.assign((size_t)G, m);
  const int64_t total = a->nnz + m;
  int64_t rb = 0;
  for (int g = 0; g < G; ++g) {
    // first row of group g + 1: cost (indptr[i] + i) reaches (g + 1) / G of the total
    const int64_t target = (total * (g + 1) + G - 1) / G;
    int64_t lo = rb, hi = m;
    while (lo < hi) {
      const int64_t mid = (lo + hi) / 2;
      if (a->indptr[mid] + mid >= target) hi = mid;
      else lo = mid + 1;
    }
    r->group_end[(size_t)g] = g == G - 1 ? m : lo;
    rb = r->group_end[(size_t)g];
  }
  // per row: owned / remote nonzeros; first_phase = 0 when segment 0 writes the row
  auto owned = [&](int64_t c) { return r->remap[(size_t)(c / r->cpt)] == me; };
  std::vector<uint8_t> fp((size_t)std::max<int64_t>(m, 1), 0xff);
  std::vector<int32_t> grp((size_t)std::max<int64_t>(m, 1), 0);
  {
    int g = 0;
    for (int64_t i = 0; i < m; ++i) {
      while (g + 1 < G && i >= r->group_end[(size_t)g]) ++g;
      grp[(size_t)i] = g;
    }
  }
  std::vector<uint8_t> has_own((size_t)std::max<int64_t>(m, 1), 0), has_rem((size_t)std::max<int64_t>(m, 1), 0);
  parallel_for(m, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i)
      for (int64_t j = a->indptr[i]; j < a->indptr[i + 1]; ++j) (owned(a->indices[j]) ? has_own : has_rem)[(size_t)i] = 1;
  }, 1024);
  int64_t own_nnz = 0;
  for (int64_t i = 0; i < m; ++i) {
    if (has_own[(size_t)i]) fp[(size_t)i] = 0;
    else if (has_rem[(size_t)i]) fp[(size_t)i] = (uint8_t)(grp[(size_t)i] + 1);
  }
  int rc = dev_upload(&r->d_first_phase, fp.data(), fp.size());
  if (rc) return rc;
  // segment k: listed rows and their nonzeros (owned ones for k = 0, group k - 1's remote ones)
  for (int k = 0; k <= G; ++k) {
    const int64_t r0 = k == 0 ? 0 : (k == 1 ? 0 : r->group_end[(size_t)k - 2]);
    const int64_t r1 = k == 0 ? m : r->group_end[(size_t)k - 1];
    std::vector<int32_t> rows;
    std::vector<int64_t> ptr(1, 0), idx;
    std::vector<float> val;
    for (int64_t i = r0; i < r1; ++i) {
      const int64_t before = (int64_t)idx.size();
      for (int64_t j = a->indptr[i]; j < a->indptr[i + 1]; ++j)
        if (owned(a->indices[j]) == (k == 0)) {
          idx.push_back(a->indices[j]);
          val.push_back(a->values[j]);
        }
      if ((int64_t)idx.size() > before) {
        rows.push_back((int32_t)i);
        ptr.push_back((int64_t)idx.size());
      }
    }
    if (k == 0) own_nnz = (int64_t)idx.size();
    auto &S = r->segs[(size_t)k];
    S.owner = k == 0 ? me : -1;
    if (idx.empty()) continue;
    rc = S.op.upload(r->device, m, r->M, ptr.data(), rows.data(), (int64_t)rows.size(), idx.data(), val.data(), 0,
                     ptr.back(), r->dims, false);
    if (rc) return rc;
    r->scratch_floats = std::max(r->scratch_floats, S.op.pieces * (int64_t)r->dims);
  }
  r->stats.phase0_nnz = own_nnz;
  return DSP_OK;
}

// Groups pipeline fetch plan: every row of a sparse tile's fetch list is fetched with the
// first group whose nonzeros use it (rows no local nonzero uses, with the last group), in
// ascending row order per (group, peer), so the rows moved are those of the other
// pipelines' plan; bulk tiles with
// local nonzeros are copied whole before group 0 (tiles without local nonzeros are
// skipped, src/dist_spmm_node.cu:344).
int build_group_fetch(dsp_rank *r, const dsp_rank_desc *d) {
  const int P = r->P, T = r->T, G = r->n_groups, me = r->me;
  const dsp_csr *a = d->local;
  std::vector<int64_t> nnz_t((size_t)T, 0);
  for (int64_t j = 0; j < a->nnz; ++j) nnz_t[(size_t)(a->indices[j] / r->cpt)]++;
  r->fetch.assign((size_t)P, dsp_rank::Fetch());
  for (int t = 0; t < T; ++t) {
    const int q = r->remap[(size_t)t];
    if (q == me || nnz_t[(size_t)t] == 0) continue;
    if (r->sparse[(size_t)t]) {
      r->stats.fetch_sparse_tiles++;
    } else {
      const int64_t row0 = (int64_t)t * r->cpt, n = std::min<int64_t>(r->cpt, r->M - row0);
      if (n > 0) r->fetch[(size_t)((q - me + P) % P)].bulk.push_back({row0, n});
      r->stats.fetch_bulk_tiles++;
      r->stats.fetch_rows += n;
    }
  }
  // first group needing each remote row of a sparse tile (groups are contiguous row ranges)
  std::vector<uint8_t> first((size_t)r->M, 0xff);
  int g = 0;
  for (int64_t i = 0; i < a->num_rows; ++i) {
    while (g + 1 < G && i >= r->group_end[(size_t)g]) ++g;
    for (int64_t j = a->indptr[i]; j < a->indptr[i + 1]; ++j) {
      const int64_t c = a->indices[j];
      const int64_t t = c / r->cpt;
      if (r->remap[(size_t)t] == me || !r->sparse[(size_t)t] || first[(size_t)c] != 0xff) continue;
      first[(size_t)c] = (uint8_t)g;
    }
  }
  // the sparse tiles' fetch lists (the rank's own needs, or the node union under the
  // reference's scope), each row in the first group that needs it; rows that no local
  // nonzero needs (other ranks' needs in a node list) go with the last group
  std::vector<std::vector<int32_t>> lists((size_t)G * P);
  for (int t = 0; t < T; ++t) {
    const int q = r->remap[(size_t)t];
    if (q == me || nnz_t[(size_t)t] == 0 || !r->sparse[(size_t)t]) continue;
    const int64_t row0 = (int64_t)t * r->cpt;
    for (int64_t p = d->needed_offsets[t]; p < d->needed_offsets[t + 1]; ++p) {
      const int64_t c = row0 + d->needed_cols[p];
      const int gg = first[(size_t)c] == 0xff ? G - 1 : first[(size_t)c];
      lists[(size_t)gg * P + (size_t)((q - me + P) % P)].push_back((int32_t)c);
    }
  }
  r->gfetch.assign((size_t)G * P, dsp_rank::Fetch());
  for (size_t i = 0; i < lists.size(); ++i) {
    auto &F = r->gfetch[i];
    F.n_rows = (int64_t)lists[i].size();
    r->stats.fetch_rows += F.n_rows;
    if (F.n_rows) {
      int rc = dev_upload(&F.d_rows, lists[i].data(), sizeof(int32_t) * lists[i].size());
      if (rc) return rc;
    }
  }
  r->stats.fetch_bytes = r->stats.fetch_rows * (int64_t)r->dims * 4;
  return DSP_OK;
}

}  // namespace

extern "C" int dsp_rank_create(const dsp_rank_desc *d, dsp_rank **out) {
  DSP_TRY_ARG(d && out && d->local && d->remap, "dsp_rank_create: null argument");
  DSP_TRY_ARG(d->world >= 1 && d->rank >= 0 && d->rank < d->world, "dsp_rank_create: rank %d of %d", d->rank,
              d->world);
  DSP_TRY_ARG(d->dims >= 1 && d->T >= 1 && d->cpt >= 1 && d->M >= 1, "dsp_rank_create: dims/T/cpt/M");
  DSP_TRY_ARG(d->M <= INT32_MAX, "dsp_rank_create: M must fit int32");
  DSP_TRY_ARG(d->local->num_cols == d->M, "dsp_rank_create: local matrix has %lld columns, M = %lld",
              (long long)d->local->num_cols, (long long)d->M);
  DSP_TRY_ARG(d->world == 1 || (d->sparse && d->needed_offsets), "dsp_rank_create: fetch plan missing");
  *out = nullptr;
  for (int t = 0; t < d->T; ++t)
    DSP_TRY_ARG(d->remap[t] >= 0 && d->remap[t] < d->world, "dsp_rank_create: remap[%d] = %d", t, d->remap[t]);
  DSP_TRY_ARG((int64_t)d->T * d->cpt >= d->M, "dsp_rank_create: T * cpt < M");
  DeviceGuard g(d->device);
  DSP_CUDA(cudaSetDevice(d->device));
  prefer_l1_carveout();
  dsp_rank *r = new dsp_rank();
  r->me = d->rank;
  r->P = d->world;
  r->device = d->device;
  r->dims = d->dims;
  r->T = d->T;
  r->n_streams = std::max(1, d->n_streams);
  r->fetch_engine = d->fetch_engine == DSP_FETCH_TMA ? DSP_FETCH_TMA : DSP_FETCH_LSU;
  r->cpt = d->cpt;
  r->M = d->M;
  r->m_lb = d->m_lb;
  r->m_local = d->local->num_rows;
  r->nnz_local = d->local->nnz;
  r->remap.assign(d->remap, d->remap + d->T);
  if (d->sparse) r->sparse.assign(d->sparse, d->sparse + d->T);
  else r->sparse.assign((size_t)d->T, 0);
  r->peer_B.assign((size_t)r->P, nullptr);
  r->peer_dev.assign((size_t)r->P, -1);
  r->peer_ipc.assign((size_t)r->P, false);
  for (int t = 0; t < d->T; ++t)
    if (r->remap[(size_t)t] == r->me) r->owned.push_back(t);

  auto bail = [&](int rc) {
    dsp_rank_destroy(r);
    return rc;
  };
  int rc;
  cudaError_t e;
  const size_t bbytes = sizeof(float) * (size_t)r->M * r->dims;
  const size_t cbytes = sizeof(float) * (size_t)std::max<int64_t>(r->m_local, 1) * r->dims;
  if ((e = cudaMalloc(&r->B, bbytes)) != cudaSuccess)
    return bail(fail(DSP_ERR_NOMEM, "B (%zu bytes): %s", bbytes, cudaGetErrorString(e)));
  if ((e = cudaMalloc(&r->C, cbytes)) != cudaSuccess)
    return bail(fail(DSP_ERR_NOMEM, "C (%zu bytes): %s", cbytes, cudaGetErrorString(e)));
  if ((e = cudaMalloc(&r->d_err, sizeof(int))) != cudaSuccess || (e = cudaMemset(r->d_err, 0, sizeof(int))) != cudaSuccess)
    return bail(fail(DSP_ERR_NOMEM, "error flag: %s", cudaGetErrorString(e)));
  if ((rc = build_phases(r, d->local, d->pipeline, d->groups, planned_fetch_rows(r, d)))) return bail(rc);
  if (r->P > 1 && (rc = r->n_groups > 0 ? build_group_fetch(r, d) : build_fetch(r, d))) return bail(rc);
  if (r->scratch_floats > 0 && (e = cudaMalloc(&r->scratch, sizeof(float) * (size_t)r->scratch_floats)) != cudaSuccess)
    return bail(fail(DSP_ERR_NOMEM, "scratch: %s", cudaGetErrorString(e)));
  int lo = 0, hi = 0;
  cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if ((e = cudaStreamCreateWithPriority(&r->compute, cudaStreamNonBlocking, lo)) != cudaSuccess ||
      (e = cudaStreamCreateWithPriority(&r->side, cudaStreamNonBlocking, hi)) != cudaSuccess)
    return bail(fail(DSP_ERR_CUDA, "stream: %s", cudaGetErrorString(e)));
  for (int i = 0; i < (r->P > 1 ? r->n_streams : 0); ++i) {
    cudaStream_t s;
    if ((e = cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, hi)) != cudaSuccess)
      return bail(fail(DSP_ERR_CUDA, "stream: %s", cudaGetErrorString(e)));
    r->fstreams.push_back(s);
  }
  if (cudaEventCreate(&r->ev_start) != cudaSuccess || cudaEventCreate(&r->ev_c0) != cudaSuccess ||
      cudaEventCreate(&r->ev_c1) != cudaSuccess ||
      cudaEventCreateWithFlags(&r->ev_zero, cudaEventDisableTiming) != cudaSuccess)
    return bail(fail(DSP_ERR_CUDA, "event create failed"));
  const int n_seg = (int)r->segs.size();
  for (auto *v : {&r->ev_fetch, &r->ev_fetch_begin, &r->ev_seg_begin, &r->ev_seg_end}) {
    const int n = (v == &r->ev_seg_begin || v == &r->ev_seg_end) ? std::max(r->P, n_seg) : r->P;
    v->assign((size_t)n, nullptr);
    for (int k = 0; k < n; ++k)
      if (cudaEventCreate(&(*v)[(size_t)k]) != cudaSuccess) return bail(fail(DSP_ERR_CUDA, "event create failed"));
  }
  r->ev_group.assign(r->gfetch.size(), nullptr);
  for (auto &ev : r->ev_group)
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess)
      return bail(fail(DSP_ERR_CUDA, "event create failed"));

  // statistics
  auto &s = r->stats;
  s.m_local = r->m_local;
  s.nnz_local = r->nnz_local;
  s.segments = 0;
  s.launches_per_step = 0;
  s.kernels_per_step = r->n_empty > 0;
  for (int k = 0; k < n_seg; ++k) {
    const auto &op = r->segs[(size_t)k].op;
    if (op.units() > 0) {
      s.segments++;
      s.kernels_per_step += 1 + (op.n_split > 0);
    }
  }
  for (int k = 1; k < r->P && k < (int)r->fetch.size(); ++k) {
    s.kernels_per_step += r->fetch[(size_t)k].n_rows > 0;
    s.launches_per_step += (int64_t)r->fetch[(size_t)k].bulk.size();
  }
  for (auto &F : r->gfetch) s.kernels_per_step += F.n_rows > 0;
  s.timeline_len = std::max(r->P, n_seg);
  s.model_rows_ms = r->model_ms[0];
  s.model_split_ms = r->model_ms[1];
  s.model_groups_ms = r->model_ms[2];
  s.launches_per_step += s.kernels_per_step;
  for (int64_t t : r->owned) s.owned_rows += std::max<int64_t>(0, std::min<int64_t>(r->cpt, r->M - t * r->cpt));
  {
    std::vector<uint8_t> seen((size_t)r->M, 0);
    for (int64_t j = 0; j < r->nnz_local; ++j) seen[(size_t)d->local->indices[j]] = 1;
    for (auto x : seen) s.distinct_cols += x;
  }
  s.pipeline = r->pipeline;
  s.device_bytes = (int64_t)bbytes + (int64_t)cbytes + r->scratch_floats * 4 +
                   (r->d_first_phase ? std::max<int64_t>(r->m_local, 1) : 0);
  for (auto &S : r->segs) s.device_bytes += S.op.device_bytes();
  for (auto &F : r->fetch) s.device_bytes += F.n_rows * 4;
  for (auto &F : r->gfetch) s.device_bytes += F.n_rows * 4;
  *out = r;
  return DSP_OK;
}

extern "C" void dsp_rank_destroy(dsp_rank *r) {
  if (!r) return;
  DeviceGuard g(r->device);
  if (r->compute) cudaStreamSynchronize(r->compute);
  if (r->side) cudaStreamSynchronize(r->side);
  for (auto s : r->fstreams) cudaStreamSynchronize(s);
  for (int p = 0; p < r->P; ++p)
    if (r->peer_ipc[(size_t)p] && r->peer_B[(size_t)p]) cudaIpcCloseMemHandle((void *)r->peer_B[(size_t)p]);
  for (auto &S : r->segs) S.op.release();
  for (auto *v : {&r->fetch, &r->gfetch})
    for (auto &F : *v)
      if (F.d_rows) cudaFree(F.d_rows);
  for (auto ev : r->ev_group)
    if (ev) cudaEventDestroy(ev);
  if (r->B) cudaFree(r->B);
  if (r->C) cudaFree(r->C);
  if (r->scratch) cudaFree(r->scratch);
  if (r->d_empty) cudaFree(r->d_empty);
  if (r->d_first_phase) cudaFree(r->d_first_phase);
  if (r->d_err) cudaFree(r->d_err);
  for (auto s : r->fstreams) cudaStreamDestroy(s);
  if (r->compute) cudaStreamDestroy(r->compute);
  if (r->side) cudaStreamDestroy(r->side);
  for (auto ev : {r->ev_start, r->ev_c0, r->ev_c1, r->ev_zero})
    if (ev) cudaEventDestroy(ev);
  for (auto *v : {&r->ev_fetch, &r->ev_fetch_begin, &r->ev_seg_begin, &r->ev_seg_end})
    for (auto ev : *v)
      if (ev) cudaEventDestroy(ev);
  cudaGetLastError();
  delete r;
}

extern "C" int dsp_rank_stats_get(const dsp_rank *r, dsp_rank_stats *s) {
  DSP_TRY_ARG(r && s, "dsp_rank_stats_get: null argument");
  *s = r->stats;
  return DSP_OK;
}

extern "C" int dsp_rank_b_ptr(dsp_rank *r, float **B) {
  DSP_TRY_ARG(r && B, "dsp_rank_b_ptr: null argument");
  *B = r->B;
  return DSP_OK;
}

extern "C" int dsp_rank_c_ptr(dsp_rank *r, float **C) {
  DSP_TRY_ARG(r && C, "dsp_rank_c_ptr: null argument");
  *C = r->C;
  return DSP_OK;
}

extern "C" int dsp_rank_ipc_handle(dsp_rank *r, void *handle64) {
  DSP_TRY_ARG(r && handle64, "dsp_rank_ipc_handle: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  DeviceGuard g(r->device);
  cudaIpcMemHandle_t h;
  DSP_CUDA(cudaIpcGetMemHandle(&h, r->B));
  memcpy(handle64, &h, sizeof h);
  return DSP_OK;
}

extern "C" int dsp_rank_open_peer(dsp_rank *r, int peer, const void *handle64) {
  DSP_TRY_ARG(r && handle64 && peer >= 0 && peer < r->P && peer != r->me, "dsp_rank_open_peer: bad argument");
  DeviceGuard g(r->device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof h);
  void *p = nullptr;
  DSP_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  r->peer_B[(size_t)peer] = (const float *)p;
  r->peer_ipc[(size_t)peer] = true;
  return DSP_OK;
}

extern "C" int dsp_rank_set_peer(dsp_rank *r, int peer, const float *peer_B, int peer_device) {
  DSP_TRY_ARG(r && peer_B && peer >= 0 && peer < r->P && peer != r->me, "dsp_rank_set_peer: bad argument");
  DeviceGuard g(r->device);
  if (peer_device >= 0 && peer_device != r->device) {
    int ok = 0;
    DSP_CUDA(cudaDeviceCanAccessPeer(&ok, r->device, peer_device));
    if (!ok) return fail(DSP_ERR_UNSUPPORTED, "device %d cannot access device %d", r->device, peer_device);
    cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
    else if (e != cudaSuccess) return fail(DSP_ERR_CUDA, "enable peer access: %s", cudaGetErrorString(e));
  }
  r->peer_B[(size_t)peer] = peer_B;
  r->peer_dev[(size_t)peer] = peer_device;
  return DSP_OK;
}

extern "C" int dsp_rank_fill_b(dsp_rank *r, uint64_t seed, void *stream) {
  DSP_TRY_ARG(r, "dsp_rank_fill_b: null rank");
  DeviceGuard g(r->device);
  for (int64_t t : r->owned) {
    const int64_t row0 = t * r->cpt, n = std::min<int64_t>(r->cpt, r->M - row0);
    if (n <= 0) continue;
    int rc = launch_fill_dense(r->B + row0 * r->dims, row0, n, r->dims, r->dims, seed, (cudaStream_t)stream);
    if (rc) return rc;
  }
  return DSP_OK;
}

extern "C" int dsp_rank_poison_remote(dsp_rank *r, void *stream) {
  DSP_TRY_ARG(r, "dsp_rank_poison_remote: null rank");
  DeviceGuard g(r->device);
  std::vector<bool> own((size_t)r->T, false);
  for (int64_t t : r->owned) own[(size_t)t] = true;
  for (int t = 0; t < r->T; ++t) {
    if (own[(size_t)t]) continue;
    const int64_t row0 = (int64_t)t * r->cpt, n = std::min<int64_t>(r->cpt, r->M - row0);
    if (n <= 0) continue;
    int rc = launch_fill_const(r->B + row0 * r->dims, n * r->dims, nanf(""), (cudaStream_t)stream);
    if (rc) return rc;
  }
  return DSP_OK;
}

extern "C" int dsp_rank_upload_b(dsp_rank *r, const float *B_host, void *stream) {
  DSP_TRY_ARG(r && B_host, "dsp_rank_upload_b: null argument");
  DeviceGuard g(r->device);
  for (int64_t t : r->owned) {
    const int64_t row0 = t * r->cpt, n = std::min<int64_t>(r->cpt, r->M - row0);
    if (n <= 0) continue;
    const size_t off = (size_t)row0 * r->dims;
    DSP_CUDA(cudaMemcpyAsync(r->B + off, B_host + off, sizeof(float) * (size_t)n * r->dims, cudaMemcpyHostToDevice,
                             (cudaStream_t)stream));
  }
  return DSP_OK;
}

extern "C" int dsp_rank_upload_b_owned(dsp_rank *r, const float *B_owned_host, void *stream) {
  DSP_TRY_ARG(r && B_owned_host, "dsp_rank_upload_b_owned: null argument");
  DeviceGuard g(r->device);
  size_t off = 0;
  for (int64_t t : r->owned) {
    const int64_t row0 = t * r->cpt, n = std::min<int64_t>(r->cpt, r->M - row0);
    if (n <= 0) continue;
    const size_t bytes = sizeof(float) * (size_t)n * r->dims;
    DSP_CUDA(cudaMemcpyAsync(r->B + (size_t)row0 * r->dims, B_owned_host + off, bytes, cudaMemcpyHostToDevice,
                             (cudaStream_t)stream));
    off += (size_t)n * r->dims;
  }
  return DSP_OK;
}

extern "C" int dsp_rank_download_c(dsp_rank *r, float *C_host, void *stream) {
  DSP_TRY_ARG(r && C_host, "dsp_rank_download_c: null argument");
  DeviceGuard g(r->device);
  if (r->m_local == 0) return DSP_OK;
  DSP_CUDA(cudaMemcpyAsync(C_host, r->C, sizeof(float) * (size_t)r->m_local * r->dims, cudaMemcpyDeviceToHost,
                           (cudaStream_t)stream));
  return DSP_OK;
}

namespace {

// One step of the groups pipeline: bulk tiles, then the fetches of group 0 from every peer,
// group 1, ... (group-major, so each fetch stream serves its peers' groups in order), while
// the compute stream runs segment 0 (owned columns) at once and group g's remote nonzeros
// once the fetches of groups 0..g have landed.
int step_groups(dsp_rank *r, cudaStream_t stream) {
  const int P = r->P, G = r->n_groups;
  for (int k = 1; k < P; ++k) {
    bool any = !r->fetch[(size_t)k].bulk.empty();
    for (int g = 0; g < G; ++g) any = any || r->gfetch[(size_t)g * P + k].n_rows > 0;
    if (any && !r->peer_B[(size_t)((r->me + k) % P)])
      return fail(DSP_ERR_STATE, "rank %d: B of peer %d not attached", r->me, (r->me + k) % P);
  }
  DSP_CUDA(cudaEventRecord(r->ev_start, stream));
  DSP_CUDA(cudaStreamWaitEvent(r->compute, r->ev_start, 0));
  for (auto s : r->fstreams) DSP_CUDA(cudaStreamWaitEvent(s, r->ev_start, 0));
  std::vector<bool> has_fetch((size_t)P, false);
  std::vector<std::vector<bool>> landed((size_t)G, std::vector<bool>((size_t)P, false));
  for (int k = 1; k < P; ++k) {  // bulk tiles first, counted as group 0's
    const auto &F = r->fetch[(size_t)k];
    cudaStream_t fs = r->fstreams[(size_t)((k - 1) % r->n_streams)];
    DSP_CUDA(cudaEventRecord(r->ev_fetch_begin[(size_t)k], fs));
    if (F.bulk.empty()) continue;
    const float *src = r->peer_B[(size_t)((r->me + k) % P)];
    for (const auto &b : F.bulk) {
      const size_t off = (size_t)b.first * r->dims;
      DSP_CUDA(cudaMemcpyAsync(r->B + off, src + off, sizeof(float) * (size_t)b.second * r->dims, cudaMemcpyDefault,
                               fs));
    }
    has_fetch[(size_t)k] = true;
  }
  for (int g = 0; g < G; ++g)
    for (int k = 1; k < P; ++k) {
      const auto &F = r->gfetch[(size_t)g * P + k];
      cudaStream_t fs = r->fstreams[(size_t)((k - 1) % r->n_streams)];
      if (F.n_rows) {
        int rc = launch_gather_rows(r->B, r->peer_B[(size_t)((r->me + k) % P)], F.d_rows, F.n_rows, r->dims,
                                    r->fetch_engine, r->d_err, fs);
        if (rc) return rc;
        has_fetch[(size_t)k] = true;
      }
      if (F.n_rows || (g == 0 && !r->fetch[(size_t)k].bulk.empty())) {
        DSP_CUDA(cudaEventRecord(r->ev_group[(size_t)g * P + k], fs));
        landed[(size_t)g][(size_t)k] = true;
      }
    }
  for (int k = 1; k < P; ++k)
    if (has_fetch[(size_t)k])
      DSP_CUDA(cudaEventRecord(r->ev_fetch[(size_t)k], r->fstreams[(size_t)((k - 1) % r->n_streams)]));
  DSP_CUDA(cudaEventRecord(r->ev_c0, r->compute));
  int rc;
  if (r->n_empty) {
    DSP_CUDA(cudaStreamWaitEvent(r->side, r->ev_c0, 0));
    if ((rc = launch_zero_rows(r->C, r->dims, r->d_empty, r->n_empty, r->dims, r->side))) return rc;
    DSP_CUDA(cudaEventRecord(r->ev_zero, r->side));
  }
  r->seg_ran.assign(r->ev_seg_begin.size(), false);
  for (int k = 0; k <= G; ++k) {  // segment 0: owned columns; segment g + 1: group g's remote ones
    if (k > 0)
      for (int q = 1; q < P; ++q)
        if (landed[(size_t)k - 1][(size_t)q])
          DSP_CUDA(cudaStreamWaitEvent(r->compute, r->ev_group[(size_t)(k - 1) * P + q], 0));
    const auto &op = r->segs[(size_t)k].op;
    if (op.units() == 0) continue;
    DSP_CUDA(cudaEventRecord(r->ev_seg_begin[(size_t)k], r->compute));
    SpmmArgs sa = op.args(r->B, r->dims, r->C, r->dims, r->dims, r->scratch);
    sa.err = r->d_err;
    sa.first_phase = r->d_first_phase;  // rows written by segment 0 are accumulated
    sa.phase = k;
    if ((rc = launch_spmm(sa, false, r->compute))) return rc;
    DSP_CUDA(cudaEventRecord(r->ev_seg_end[(size_t)k], r->compute));
    r->seg_ran[(size_t)k] = true;
  }
  r->fetch_ran = has_fetch;
  if (r->n_empty) DSP_CUDA(cudaStreamWaitEvent(r->compute, r->ev_zero, 0));
  DSP_CUDA(cudaEventRecord(r->ev_c1, r->compute));
  for (int k = 1; k < P; ++k)
    if (has_fetch[(size_t)k]) DSP_CUDA(cudaStreamWaitEvent(stream, r->ev_fetch[(size_t)k], 0));
  DSP_CUDA(cudaStreamWaitEvent(stream, r->ev_c1, 0));
  return DSP_OK;
}

}  // namespace

extern "C" int dsp_rank_step(dsp_rank *r, void *stream_v) {
  DSP_TRY_ARG(r, "dsp_rank_step: null rank");
  DeviceGuard g(r->device);
  cudaStream_t stream = (cudaStream_t)stream_v;
  if (r->n_groups > 0) return step_groups(r, stream);
  for (int k = 1; k < r->P; ++k) {
    const auto &F = r->fetch[(size_t)k];
    if ((F.n_rows || !F.bulk.empty()) && !r->peer_B[(size_t)r->segs[(size_t)k].owner])
      return fail(DSP_ERR_STATE, "rank %d: B of peer %d not attached", r->me, r->segs[(size_t)k].owner);
  }
  DSP_CUDA(cudaEventRecord(r->ev_start, stream));
  DSP_CUDA(cudaStreamWaitEvent(r->compute, r->ev_start, 0));
  for (auto s : r->fstreams) DSP_CUDA(cudaStreamWaitEvent(s, r->ev_start, 0));
  // fetch: peers in ring order, spread over the fetch streams
  std::vector<bool> has_fetch((size_t)r->P, false);
  for (int k = 1; k < r->P; ++k) {
    const auto &F = r->fetch[(size_t)k];
    if (!F.n_rows && F.bulk.empty()) continue;
    cudaStream_t fs = r->fstreams[(size_t)((k - 1) % r->n_streams)];
    const float *src = r->peer_B[(size_t)r->segs[(size_t)k].owner];
    DSP_CUDA(cudaEventRecord(r->ev_fetch_begin[(size_t)k], fs));
    for (const auto &b : F.bulk) {
      const size_t off = (size_t)b.first * r->dims;
      DSP_CUDA(cudaMemcpyAsync(r->B + off, src + off, sizeof(float) * (size_t)b.second * r->dims, cudaMemcpyDefault,
                               fs));
    }
    int rc = launch_gather_rows(r->B, src, F.d_rows, F.n_rows, r->dims, r->fetch_engine, r->d_err, fs);
    if (rc) return rc;
    DSP_CUDA(cudaEventRecord(r->ev_fetch[(size_t)k], fs));
    has_fetch[(size_t)k] = true;
  }
  // compute: phase k once the fetches of ring positions 1..k landed; the empty rows (other
  // rows of C) are zero-filled beside them on the side stream
  DSP_CUDA(cudaEventRecord(r->ev_c0, r->compute));
  int rc;
  if (r->n_empty) {
    DSP_CUDA(cudaStreamWaitEvent(r->side, r->ev_c0, 0));
    if ((rc = launch_zero_rows(r->C, r->dims, r->d_empty, r->n_empty, r->dims, r->side))) return rc;
    DSP_CUDA(cudaEventRecord(r->ev_zero, r->side));
  }
  r->seg_ran.assign((size_t)r->P, false);
  int waited = 0;
  for (int k = 0; k < r->P; ++k) {
    const auto &op = r->segs[(size_t)k].op;
    if (op.units() == 0) continue;
    for (; waited < k; ++waited)
      if (has_fetch[(size_t)waited + 1]) DSP_CUDA(cudaStreamWaitEvent(r->compute, r->ev_fetch[(size_t)waited + 1], 0));
    DSP_CUDA(cudaEventRecord(r->ev_seg_begin[(size_t)k], r->compute));
    SpmmArgs sa = op.args(r->B, r->dims, r->C, r->dims, r->dims, r->scratch);
    sa.err = r->d_err;
    if (r->pipeline == DSP_PIPELINE_SPLIT) {  // rows written by an earlier phase are accumulated
      sa.first_phase = r->d_first_phase;
      sa.phase = k;
    }
    if ((rc = launch_spmm(sa, false, r->compute))) return rc;
    DSP_CUDA(cudaEventRecord(r->ev_seg_end[(size_t)k], r->compute));
    r->seg_ran[(size_t)k] = true;
  }
  r->fetch_ran = has_fetch;
  if (r->n_empty) DSP_CUDA(cudaStreamWaitEvent(r->compute, r->ev_zero, 0));
  DSP_CUDA(cudaEventRecord(r->ev_c1, r->compute));
  for (int k = 1; k < r->P; ++k)
    if (has_fetch[(size_t)k]) DSP_CUDA(cudaStreamWaitEvent(stream, r->ev_fetch[(size_t)k], 0));
  DSP_CUDA(cudaStreamWaitEvent(stream, r->ev_c1, 0));
  return DSP_OK;
}

extern "C" int dsp_rank_check_error(dsp_rank *r) {
  DSP_TRY_ARG(r, "dsp_rank_check_error: null rank");
  DeviceGuard g(r->device);
  int flag = 0;
  DSP_CUDA(cudaMemcpy(&flag, r->d_err, sizeof flag, cudaMemcpyDeviceToHost));
  if (flag == 0) return DSP_OK;
  DSP_CUDA(cudaMemset(r->d_err, 0, sizeof(int)));
  return fail(DSP_ERR_TIMEOUT, "rank %d: a fetch wait gave up (code %d); the step's C is incomplete", r->me, flag);
}

extern "C" int dsp_rank_last_compute_ms(dsp_rank *r, float *ms) {
  DSP_TRY_ARG(r && ms, "dsp_rank_last_compute_ms: null argument");
  DeviceGuard g(r->device);
  DSP_CUDA(cudaEventElapsedTime(ms, r->ev_c0, r->ev_c1));
  return DSP_OK;
}

extern "C" int dsp_rank_last_timeline(dsp_rank *r, float *ms, int cap) {
  const int n = r ? (int)r->stats.timeline_len : 0;
  DSP_TRY_ARG(r && ms && cap >= 4 * n, "dsp_rank_last_timeline: need %d floats", 4 * n);
  DeviceGuard g(r->device);
  for (int k = 0; k < n; ++k) {
    float *o = ms + 4 * k;
    o[0] = o[1] = o[2] = o[3] = -1.f;
    if (k < (int)r->fetch_ran.size() && r->fetch_ran[(size_t)k]) {
      DSP_CUDA(cudaEventElapsedTime(&o[0], r->ev_start, r->ev_fetch_begin[(size_t)k]));
      DSP_CUDA(cudaEventElapsedTime(&o[1], r->ev_start, r->ev_fetch[(size_t)k]));
    }
    if (k < (int)r->seg_ran.size() && r->seg_ran[(size_t)k]) {
      DSP_CUDA(cudaEventElapsedTime(&o[2], r->ev_start, r->ev_seg_begin[(size_t)k]));
      DSP_CUDA(cudaEventElapsedTime(&o[3], r->ev_start, r->ev_seg_end[(size_t)k]));
    }
  }
  return DSP_OK;
}
