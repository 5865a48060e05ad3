// host_plan.cpp — integer planning of the distributed SpMM, bit-exact with the reference:
// column tiling and needed sets, HSDMA tile allocation, node-level merge, the adaptive
// bulk/sparse selector and the traffic formulas; plus the work-item builder of the SpMM
// kernels.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "internal.h"

using namespace dsp;

namespace {

// Column bitmap helpers (one bit per global column).
inline void bit_set_atomic(uint64_t *bm, int64_t c) {
  __atomic_fetch_or(&bm[c >> 6], 1ull << (c & 63), __ATOMIC_RELAXED);
}

// Number of set bits in [lo, hi).
int64_t bit_count(const uint64_t *bm, int64_t lo, int64_t hi) {
  if (lo >= hi) return 0;
  int64_t n = 0;
  int64_t wlo = lo >> 6, whi = (hi - 1) >> 6;
  for (int64_t w = wlo; w <= whi; ++w) {
    uint64_t x = bm[w];
    if (w == wlo) x &= ~0ull << (lo & 63);
    if (w == whi && (hi & 63)) x &= (1ull << (hi & 63)) - 1;
    n += __builtin_popcountll(x);
  }
  return n;
}

// Append (c - base) for every set bit c in [lo, hi), ascending.
void bit_list(const uint64_t *bm, int64_t lo, int64_t hi, int64_t base, int32_t *out) {
  if (lo >= hi) return;
  int64_t wlo = lo >> 6, whi = (hi - 1) >> 6;
  for (int64_t w = wlo; w <= whi; ++w) {
    uint64_t x = bm[w];
    if (w == wlo) x &= ~0ull << (lo & 63);
    if (w == whi && (hi & 63)) x &= (1ull << (hi & 63)) - 1;
    while (x) {
      int b = __builtin_ctzll(x);
      *out++ = (int32_t)((w << 6) + b - base);
      x &= x - 1;
    }
  }
}

// Bitmap of the distinct columns of a CSR.
std::vector<uint64_t> column_bitmap(const dsp_csr *a) {
  std::vector<uint64_t> bm((size_t)((a->num_cols + 63) / 64) + 1, 0);
  parallel_for(a->nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j) bit_set_atomic(bm.data(), a->indices[j]);
  }, 1 << 16);
  return bm;
}

int check_tiling(const dsp_csr *local, int T) {
  DSP_TRY_ARG(local && local->indptr, "tiling: null matrix");
  DSP_TRY_ARG(T >= 1, "tiling: T = %d", T);
  DSP_TRY_ARG(local->num_cols >= 1, "tiling: no columns");
  DSP_TRY_ARG((local->num_cols + T - 1) / T <= INT32_MAX, "tiling: tile too tall for int32 ids");
  return DSP_OK;
}

}  // namespace

// ----------------------------------------------------------------- tiling

extern "C" int dsp_tile_counts(const dsp_csr *local, int T, int64_t *cpt_out, int32_t *n_col_list,
                               int32_t *n_slice_list, int64_t *nnz_list) {
  int rc = check_tiling(local, T);
  if (rc) return rc;
  const int64_t N = local->num_cols;
  const int64_t cpt = (N + T - 1) / T;  // src/dist_spmm_node.cu:106
  if (cpt_out) *cpt_out = cpt;
  std::vector<int64_t> nnz_t((size_t)T, 0);
  {
    int nt = host_threads();
    std::vector<std::vector<int64_t>> part((size_t)nt, std::vector<int64_t>((size_t)T, 0));
    std::atomic<int> next{0};
    parallel_for(local->nnz, [&](int64_t b, int64_t e) {
      int me = next.fetch_add(1);
      auto &h = part[(size_t)me];
      for (int64_t j = b; j < e; ++j) h[(size_t)(local->indices[j] / cpt)]++;
    }, 1 << 16);
    for (auto &h : part)
      for (int t = 0; t < T; ++t) nnz_t[(size_t)t] += h[(size_t)t];
  }
  std::vector<uint64_t> bm;
  if (n_col_list) bm = column_bitmap(local);
  for (int t = 0; t < T; ++t) {
    int64_t lo = (int64_t)t * cpt, hi = std::min<int64_t>(lo + cpt, N);
    if (nnz_list) nnz_list[t] = nnz_t[(size_t)t];
    if (n_col_list) n_col_list[t] = (int32_t)bit_count(bm.data(), lo, hi);
    // n_slice_list is only assigned for tiles holding local nonzeros
    // (src/dist_spmm_node.cu:214, :223); it stays 0 elsewhere (:210).
    if (n_slice_list) n_slice_list[t] = nnz_t[(size_t)t] > 0 ? (int32_t)std::min<int64_t>(cpt, N - lo) : 0;
  }
  return DSP_OK;
}

extern "C" int dsp_tile_needed(const dsp_csr *local, int T, int64_t *offsets, int32_t *cols) {
  int rc = check_tiling(local, T);
  if (rc) return rc;
  DSP_TRY_ARG(offsets, "dsp_tile_needed: offsets is NULL");
  const int64_t N = local->num_cols;
  const int64_t cpt = (N + T - 1) / T;
  std::vector<uint64_t> bm = column_bitmap(local);
  offsets[0] = 0;
  for (int t = 0; t < T; ++t) {
    int64_t lo = (int64_t)t * cpt, hi = std::min<int64_t>(lo + cpt, N);
    offsets[t + 1] = offsets[t] + bit_count(bm.data(), lo, hi);
  }
  if (cols) {
    parallel_for(T, [&](int64_t b, int64_t e) {
      for (int64_t t = b; t < e; ++t) {
        int64_t lo = t * cpt, hi = std::min<int64_t>(lo + cpt, N);
        bit_list(bm.data(), lo, hi, lo, cols + offsets[t]);
      }
    }, 1);
  }
  return DSP_OK;
}

// ----------------------------------------------------------------- HSDMA

namespace {

// Greedy best-swap refinement over a units x ntask cost matrix (row-major doubles):
// up to `iters` rounds; each round scans pairs a < b on different units in lexicographic
// order, keeps the first pair with the strictly largest positive gain
// (D[ma][b] + D[mb][a]) - (D[ma][a] + D[mb][b]) and swaps their units
// (src/h_sdma.h:27-38, :129-157, :191-220).
void refine_swaps(const std::vector<double> &D, int ntask, std::vector<int> &map, int iters) {
  for (int it = 0; it < iters; ++it) {
    double best = 0;
    int ba = -1, bb = -1;
    for (int a = 0; a < ntask; ++a) {
      const int ma = map[(size_t)a];
      const double *Da = &D[(size_t)ma * ntask];
      for (int b = a + 1; b < ntask; ++b) {
        const int mb = map[(size_t)b];
        if (ma == mb) continue;
        const double *Db = &D[(size_t)mb * ntask];
        double gain = (Da[b] + Db[a]) - (Da[a] + Db[b]);
        if (gain > best) {
          best = gain;
          ba = a;
          bb = b;
        }
      }
    }
    if (!(best > 0)) break;
    std::swap(map[(size_t)ba], map[(size_t)bb]);
  }
}

}  // namespace

extern "C" int dsp_hsdma(const int32_t *demand, int P, int T, const int32_t *node_of_gpu, int tasks_per_gpu,
                         int max_inter, int max_intra, int32_t *remap) {
  DSP_TRY_ARG(demand && node_of_gpu && remap, "dsp_hsdma: null argument");
  DSP_TRY_ARG(P >= 1 && T >= 1 && tasks_per_gpu >= 1, "dsp_hsdma: P=%d T=%d tasks_per_gpu=%d", P, T,
              tasks_per_gpu);
  int nodes = 0;
  for (int g = 0; g < P; ++g) {
    DSP_TRY_ARG(node_of_gpu[g] >= 0, "dsp_hsdma: negative node id");
    nodes = std::max(nodes, node_of_gpu[g] + 1);
  }
  const int tasks_per_node = T / nodes;
  const int gpn = P / nodes;
  DSP_TRY_ARG(tasks_per_node >= 1 && gpn >= 1, "dsp_hsdma: %d nodes for %d ranks / %d tasks", nodes, P, T);
  // Phase 1 (multi-node): node demand = sum of its GPUs' rows; start from blocks of
  // tasks_per_node tasks per node (src/h_sdma.h:107-162).
  std::vector<int> node_map((size_t)T, 0);
  if (nodes > 1) {
    std::vector<double> ND((size_t)nodes * T, 0.0);
    for (int g = 0; g < P; ++g)
      for (int t = 0; t < T; ++t) ND[(size_t)node_of_gpu[g] * T + t] += demand[(size_t)g * T + t];
    for (int t = 0; t < T; ++t) node_map[(size_t)t] = t / tasks_per_node;
    refine_swaps(ND, T, node_map, max_inter);
  }
  // Phase 2: per node, its tasks ascending; start from blocks of tasks_per_gpu; refine on
  // the node's GPU rows (src/h_sdma.h:164-227).
  for (int t = 0; t < T; ++t) remap[t] = -1;
  for (int node = 0; node < nodes; ++node) {
    std::vector<int> tasks;
    for (int t = 0; t < T; ++t)
      if (node_map[(size_t)t] == node) tasks.push_back(t);
    const int n = (int)tasks.size();
    if (n == 0) continue;
    std::vector<double> GD((size_t)gpn * n);
    for (int i = 0; i < gpn; ++i)
      for (int j = 0; j < n; ++j) GD[(size_t)i * n + j] = demand[(size_t)(i + node * gpn) * T + tasks[(size_t)j]];
    std::vector<int> gmap((size_t)n);
    for (int i = 0; i < n; ++i) gmap[(size_t)i] = i / tasks_per_gpu;
    for (int i = 0; i < n; ++i)
      if (gmap[(size_t)i] >= gpn)
        return fail(DSP_ERR_INVALID, "dsp_hsdma: node %d has %d tasks for %d GPUs x %d", node, n, gpn,
                    tasks_per_gpu);
    refine_swaps(GD, n, gmap, max_intra);
    for (int i = 0; i < n; ++i) remap[tasks[(size_t)i]] = gmap[(size_t)i] + node * gpn;
  }
  return DSP_OK;
}

extern "C" int dsp_alloc_slice(int P, int n_rolls, int32_t *remap) {
  DSP_TRY_ARG(remap && P >= 1 && n_rolls >= 1, "dsp_alloc_slice: bad argument");
  for (int t = 0; t < P * n_rolls; ++t) remap[t] = t / n_rolls;
  return DSP_OK;
}

extern "C" int dsp_alloc_random(int P, int n_rolls, uint64_t seed, int32_t *remap) {
  int rc = dsp_alloc_slice(P, n_rolls, remap);
  if (rc) return rc;
  const int T = P * n_rolls;
  for (int i = T - 1; i > 0; --i) {
    int j = (int)(hash3(seed, 0x52414E44ull, (uint64_t)i) % (uint64_t)(i + 1));
    std::swap(remap[i], remap[j]);
  }
  return DSP_OK;
}

// ----------------------------------------------------------------- node merge

extern "C" int dsp_merge_needed(int R, int T, const int32_t *counts, const int32_t *cols, int64_t *merged_offsets,
                                int32_t *merged_cols, int32_t *n_col_merged) {
  DSP_TRY_ARG(R >= 1 && T >= 1 && counts && merged_offsets && n_col_merged, "dsp_merge_needed: bad argument");
  // locate every (rank, tile) list inside the flat Allgatherv layout
  std::vector<int64_t> start((size_t)R * T + 1, 0);
  int64_t cpt_hint = 0;
  for (int64_t i = 0; i < (int64_t)R * T; ++i) {
    DSP_TRY_ARG(counts[i] >= 0, "dsp_merge_needed: negative count");
    start[(size_t)i + 1] = start[(size_t)i] + counts[i];
  }
  DSP_TRY_ARG(start[(size_t)R * T] == 0 || cols, "dsp_merge_needed: cols is NULL");
  for (int64_t k = 0; k < start[(size_t)R * T]; ++k) {
    DSP_TRY_ARG(cols[k] >= 0, "dsp_merge_needed: negative column id");
    cpt_hint = std::max<int64_t>(cpt_hint, (int64_t)cols[k] + 1);
  }
  const int64_t words = (cpt_hint + 63) / 64 + 1;
  std::vector<int64_t> tile_n((size_t)T, 0);
  std::vector<std::vector<uint64_t>> bms((size_t)T);
  parallel_for(T, [&](int64_t b, int64_t e) {
    for (int64_t t = b; t < e; ++t) {
      auto &bm = bms[(size_t)t];
      bm.assign((size_t)words, 0);
      for (int r = 0; r < R; ++r) {
        const int64_t s = start[(size_t)r * T + t], f = start[(size_t)r * T + t + 1];
        for (int64_t k = s; k < f; ++k) bm[(size_t)(cols[k] >> 6)] |= 1ull << (cols[k] & 63);
      }
      tile_n[(size_t)t] = bit_count(bm.data(), 0, words * 64);
    }
  }, 1);
  merged_offsets[0] = 0;
  for (int t = 0; t < T; ++t) {
    n_col_merged[t] = (int32_t)tile_n[(size_t)t];
    merged_offsets[t + 1] = merged_offsets[t] + tile_n[(size_t)t];
  }
  if (merged_cols) {
    parallel_for(T, [&](int64_t b, int64_t e) {
      for (int64_t t = b; t < e; ++t) bit_list(bms[(size_t)t].data(), 0, words * 64, 0, merged_cols + merged_offsets[t]);
    }, 1);
  }
  return DSP_OK;
}

// ----------------------------------------------------------------- selector

extern "C" int dsp_comm_model_preset(int platform, int tier, dsp_comm_model *out) {
  DSP_TRY_ARG(out && (tier == DSP_TIER_INTRA || tier == DSP_TIER_INTER), "dsp_comm_model_preset: bad argument");
  // The reference declares these as float variables initialised from the decimal
  // literals below (src/comm_man.h:389-394); the double -> float conversion is kept.
  double p[4];
  if (platform == DSP_PLATFORM_H100) {
    const double intra[4] = {12873.61472, 125.27085, 105.50392, -4.65};
    const double inter[4] = {1452.17110, -1407.82558, 47.34021, -1.00};
    memcpy(p, tier == DSP_TIER_INTRA ? intra : inter, sizeof p);
  } else if (platform == DSP_PLATFORM_A800) {
    const double intra[4] = {4075.35, 119.61, 98.21, -3.78};
    const double inter[4] = {1440.80, -1394.99, 43.65, -1.00};
    memcpy(p, tier == DSP_TIER_INTRA ? intra : inter, sizeof p);
  } else if (platform == DSP_PLATFORM_B200) {
    // Intra: fit (distspmm_b200.fit_comm_model) of the critical densities measured by
    // distspmm_b200.comm_test between two B200s over NVLink 5 (N = 400k, 1000k, 1400k,
    // 1800k; dims 1..1024): the sparse gather wins up to ~0.9 density from 128 columns on.
    // Inter: the InfiniBand tier cannot be measured on one 8-GPU box; H100's constants.
    const double intra[4] = {0.03045, 100.87679, 130.98926, 0.49};
    const double inter[4] = {1452.17110, -1407.82558, 47.34021, -1.00};
    memcpy(p, tier == DSP_TIER_INTRA ? intra : inter, sizeof p);
  } else {
    return fail(DSP_ERR_INVALID, "dsp_comm_model_preset: unknown platform %d", platform);
  }
  out->a = (float)p[0];
  out->b = (float)p[1];
  out->c = (float)p[2];
  out->u = (float)p[3];
  return DSP_OK;
}

namespace {
// 1 / (a * k^u + b / k), k = min(c, dims), all in float (src/comm_man.h:396-400).
float model_threshold(const dsp_comm_model &m, int dims) {
  float k = std::min(m.c, (float)dims);
  float t1 = m.a * powf(k, m.u);
  float t2 = m.b / k;
  float den = t1 + t2;
  return 1.0f / den;
}
}  // namespace

extern "C" int dsp_comm_select(int comm_type, int dims, const dsp_comm_model *intra, const dsp_comm_model *inter,
                               int T, const int32_t *n_col, const int32_t *n_slice, uint8_t *sparse_intra,
                               uint8_t *sparse_inter) {
  DSP_TRY_ARG(T >= 0 && sparse_intra, "dsp_comm_select: bad argument");
  if (comm_type == 0 || comm_type == 1) {
    for (int i = 0; i < T; ++i) {
      sparse_intra[i] = (uint8_t)comm_type;
      if (sparse_inter) sparse_inter[i] = (uint8_t)comm_type;
    }
    return DSP_OK;
  }
  if (comm_type != 2) return fail(DSP_ERR_INVALID, "dsp_comm_select: comm_type %d (expected 0, 1 or 2)", comm_type);
  DSP_TRY_ARG(intra && n_col && n_slice, "dsp_comm_select: adaptive mode needs models and counts");
  DSP_TRY_ARG(!sparse_inter || inter, "dsp_comm_select: inter model missing");
  const float thr_intra = model_threshold(*intra, dims);
  const float thr_inter = sparse_inter ? model_threshold(*inter, dims) : 0.0f;
  for (int i = 0; i < T; ++i) {
    float d = (float)n_col[i] / (float)(n_slice[i] + 1);  // src/comm_man.h:402
    sparse_intra[i] = thr_intra > d;
    if (sparse_inter) sparse_inter[i] = thr_inter > d;
  }
  return DSP_OK;
}

// ----------------------------------------------------------------- traffic and rate

extern "C" int dsp_traffic_intra(int me, int T, const int32_t *remap, const uint8_t *sparse, const int32_t *n_col,
                                 const int32_t *n_slice, int dims, int64_t *bytes) {
  DSP_TRY_ARG(remap && sparse && n_col && n_slice && bytes && T >= 0, "dsp_traffic_intra: bad argument");
  int64_t b = 0;
  for (int i = 0; i < T; ++i)
    if (remap[i] != me) b += (int64_t)sizeof(float) * dims * (sparse[i] ? n_col[i] : n_slice[i]);
  *bytes = b;
  return DSP_OK;
}

extern "C" int dsp_traffic_inter(int me, int ranks_per_node, int num_nodes, int T, const int32_t *remap,
                                 const uint8_t *sparse_inter, const int32_t *n_col, const int32_t *n_slice, int dims,
                                 int64_t *bytes) {
  DSP_TRY_ARG(remap && sparse_inter && n_col && n_slice && bytes && ranks_per_node >= 1 && num_nodes >= 1,
              "dsp_traffic_inter: bad argument");
  *bytes = 0;
  if (num_nodes < 2) return DSP_OK;  // src/comm_man.h:510-512
  const int my_node = me / ranks_per_node, me_in_node = me % ranks_per_node;
  int64_t b = 0;
  // tiles owned by the same-position rank of every other node, in tile order
  // (task_assignments[remote_pe], src/comm_man.h:513-525)
  for (int node = 0; node < num_nodes; ++node) {
    if (node == my_node) continue;
    const int pe = node * ranks_per_node + me_in_node;
    for (int t = 0; t < T; ++t)
      if (remap[t] == pe) b += (int64_t)sizeof(float) * dims * (sparse_inter[t] ? n_col[t] : n_slice[t]);
  }
  *bytes = b;
  return DSP_OK;
}

extern "C" double dsp_gflops(int64_t nnz, int dims, double avg_ms) { return 2.0 * (double)nnz * dims / avg_ms / 1e6; }

// ----------------------------------------------------------------- SpMM work items

namespace dsp {

int64_t default_piece_cap(int dims) {
  int64_t cap = 32768 / std::max(dims, 1);
  cap = std::max<int64_t>(32, std::min<int64_t>(cap, 4096));
  return cap & ~int64_t(31);
}

void build_items(int64_t m, const int32_t *rows, const int64_t *row_ptr, int64_t piece_cap, bool include_empty,
                 ItemPlan *out) {
  out->item_ptr.clear();
  out->item_out.clear();
  out->split_row.clear();
  out->split_ptr.assign(1, 0);
  out->piece_cap = piece_cap;
  out->max_row_len = 0;
  out->item_ptr.reserve((size_t)m + 1);
  out->item_out.reserve((size_t)m);
  int32_t slots = 0;
  for (int64_t i = 0; i < m; ++i) {
    const int64_t b = row_ptr[i], e = row_ptr[i + 1], len = e - b;
    const int32_t row = rows ? rows[i] : (int32_t)i;
    out->max_row_len = std::max(out->max_row_len, len);
    if (len == 0 && !include_empty) continue;
    if (len <= piece_cap) {
      out->item_ptr.push_back(b);
      out->item_out.push_back(row);
      continue;
    }
    // heavy row: k balanced pieces, partial sums in consecutive slots
    const int64_t k = (len + piece_cap - 1) / piece_cap;
    for (int64_t p = 0; p < k; ++p) {
      out->item_ptr.push_back(b + len * p / k);
      out->item_out.push_back(-(slots + (int32_t)p) - 1);
    }
    slots += (int32_t)k;
    out->split_row.push_back(row);
    out->split_ptr.push_back(slots);
  }
  out->item_ptr.push_back(m > 0 ? row_ptr[m] : 0);
  // an item list that skipped trailing empty rows still ends at the last nonzero
  out->pieces = slots;
}

int64_t default_chunk_nnz(int dims, int64_t nnz) {
  static const int64_t forced = [] {
    const char *e = getenv("DSP_SPMM_CHUNK");
    return e ? (int64_t)atoll(e) : 0;
  }();
  if (forced > 0) return (forced + 31) & ~int64_t(31);
  // about 32K multiply-adds per chunk (256 nonzeros at N = 128) ...
  int64_t c = 32768 / std::max(dims, 1);
  c = std::max<int64_t>(32, std::min<int64_t>(c, 1024));
  // ... but at least ~16K chunks (enough lane groups for every SM) when the matrix allows
  const int64_t min_chunks = 16384;
  if (nnz / c < min_chunks) c = std::max<int64_t>(32, nnz / min_chunks);
  return (c + 31) & ~int64_t(31);
}

void build_chunks(int64_t m, const int32_t *rows, const int64_t *row_ptr, int64_t chunk_nnz, ChunkPlan *out) {
  const int64_t nnz = m > 0 ? row_ptr[m] : 0;
  out->chunk_nnz = chunk_nnz;
  out->n_chunks = (nnz + chunk_nnz - 1) / chunk_nnz;
  out->coo_row.assign((size_t)std::max<int64_t>(nnz, 1), 0);
  out->chunk_slot.assign((size_t)std::max<int64_t>(2 * out->n_chunks, 1), -1);
  out->split_row.clear();
  out->split_ptr.assign(1, 0);
  std::atomic<int64_t> maxlen{0};
  parallel_for(m, [&](int64_t b, int64_t e) {
    int64_t ml = 0;
    for (int64_t i = b; i < e; ++i) {
      const int32_t r = rows ? rows[i] : (int32_t)i;
      for (int64_t p = row_ptr[i]; p < row_ptr[i + 1]; ++p) out->coo_row[(size_t)p] = r;
      ml = std::max(ml, row_ptr[i + 1] - row_ptr[i]);
    }
    int64_t cur = maxlen.load();
    while (ml > cur && !maxlen.compare_exchange_weak(cur, ml)) {
    }
  }, 4096);
  out->max_row_len = maxlen.load();
  // index of the (nonempty) row holding nonzero p
  auto row_of = [&](int64_t p) { return (int64_t)(std::upper_bound(row_ptr, row_ptr + m + 1, p) - row_ptr) - 1; };
  int64_t last_idx = -1;
  int32_t slots = 0;
  auto add_slot = [&](int64_t idx) {
    if (idx != last_idx) {
      out->split_row.push_back(rows ? rows[idx] : (int32_t)idx);
      out->split_ptr.push_back(slots);
      last_idx = idx;
    }
    out->split_ptr.back() = ++slots;
    return slots - 1;
  };
  for (int64_t c = 0; c < out->n_chunks; ++c) {
    const int64_t s = c * chunk_nnz, e = std::min(s + chunk_nnz, nnz);
    const int64_t hr = row_of(s), tr = row_of(e - 1);
    const bool head_cut = row_ptr[hr] < s;        // the row began in an earlier chunk
    const bool tail_cut = row_ptr[tr + 1] > e;    // the row goes on in a later chunk
    if (hr == tr) {
      if (head_cut || tail_cut) out->chunk_slot[(size_t)(2 * c)] = out->chunk_slot[(size_t)(2 * c + 1)] = add_slot(hr);
    } else {
      if (head_cut) out->chunk_slot[(size_t)(2 * c)] = add_slot(hr);
      if (tail_cut) out->chunk_slot[(size_t)(2 * c + 1)] = add_slot(tr);
    }
  }
  out->slots = slots;
}

int choose_variant(int64_t m, const int64_t *row_ptr, int dims) {
  static const int forced = [] {
    const char *e = getenv("DSP_SPMM_VARIANT");
    if (!e) return -1;
    return strcmp(e, "rows") == 0 ? 0 : strcmp(e, "nnz") == 0 ? 1 : -1;
  }();
  if (forced >= 0) return forced;
  (void)dims;
  // Row-split keeps one row per warp: good when rows are long enough to keep several
  // B-row loads in flight and of similar length; otherwise chunks of equal nonzeros.
  int64_t nonempty = 0, maxlen = 0, nnz = m > 0 ? row_ptr[m] : 0;
  for (int64_t i = 0; i < m; ++i) {
    const int64_t len = row_ptr[i + 1] - row_ptr[i];
    nonempty += len > 0;
    maxlen = std::max(maxlen, len);
  }
  if (nonempty == 0) return 0;
  const double mean = (double)nnz / (double)nonempty;
  const double empty_frac = 1.0 - (double)nonempty / (double)m;
  return (mean >= 16.0 && (double)maxlen <= 4.0 * mean && empty_frac < 0.05) ? 0 : 1;
}

}  // namespace dsp
