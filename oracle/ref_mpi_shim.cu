// ref_mpi_shim.cu — the reference's MPI-bound host functions, run with threads as ranks.
//
// TEST INFRASTRUCTURE ONLY (never linked into the product). Built by oracle/Makefile from
// the reference sources (REF_SRC) into oracle/_ref/libdsp_ref_mpi.so, against the
// single-process MPI / NVSHMEM stand-ins in oracle/mpi_stub/ (no MPI library exists here).
// It runs the reference's own code for
//   ref_node_merge -> double_level_comm_node_processing (src/utils.h:439-547)
//   ref_hsdma_mpi  -> ComputeAllocation_HSDMA_MPI       (src/utils.h:358-437)
// on P threads (one per rank of one node) so the restatements in oracle.c and the engine's
// planner can be pinned to it (tests/golden/merge_cases.json, hsdma_mpi_cases.json).
#include <algorithm>
#include <cstdint>
#include <numeric>
#include <unordered_set>
#include <vector>

#include "utils.h"

extern "C" {

// Rank p's pre-merge needed sets: counts n_col[p*T + t] and the ids (tile-local, any order)
// in `flat`, rank-major then tile-major. Every rank runs the reference's merge; the call
// checks that all ranks end with the same n_col_list and sets, then returns the merged
// counts and (when `sorted` is not null) each tile's set in ascending order at off[t].
// Returns 0, or -1 when the ranks disagree.
int ref_node_merge(int P, int T, const int32_t *n_col, const int32_t *flat, int32_t *merged_count, int64_t *off,
                   int32_t *sorted) {
  std::vector<std::vector<int>> counts((size_t)P, std::vector<int>((size_t)T));
  std::vector<std::vector<std::vector<int>>> sets((size_t)P);
  int64_t pos = 0;
  for (int p = 0; p < P; ++p) {
    sets[(size_t)p].resize((size_t)T);
    for (int t = 0; t < T; ++t) {
      counts[(size_t)p][(size_t)t] = n_col[(size_t)p * T + t];
      sets[(size_t)p][(size_t)t].assign(flat + pos, flat + pos + n_col[(size_t)p * T + t]);
      pos += n_col[(size_t)p * T + t];
    }
  }
  std::vector<std::vector<int>> out_counts((size_t)P);
  std::vector<std::vector<std::vector<int>>> out_sets((size_t)P);
  dsp_mpi_stub::run_ranks(P, [&](int p) {
    MPI_Comm comm = MPI_COMM_WORLD;
    std::vector<int> n_col_list = counts[(size_t)p];
    std::vector<std::unordered_set<int>> col_ind_unique((size_t)T);
    for (int t = 0; t < T; ++t)
      col_ind_unique[(size_t)t].insert(sets[(size_t)p][(size_t)t].begin(), sets[(size_t)p][(size_t)t].end());
    double_level_comm_node_processing(comm, n_col_list, col_ind_unique, false);
    out_counts[(size_t)p] = n_col_list;
    out_sets[(size_t)p].resize((size_t)T);
    for (int t = 0; t < T; ++t) {
      out_sets[(size_t)p][(size_t)t].assign(col_ind_unique[(size_t)t].begin(), col_ind_unique[(size_t)t].end());
      std::sort(out_sets[(size_t)p][(size_t)t].begin(), out_sets[(size_t)p][(size_t)t].end());
    }
  });
  for (int p = 1; p < P; ++p)
    if (out_counts[(size_t)p] != out_counts[0] || out_sets[(size_t)p] != out_sets[0]) return -1;
  off[0] = 0;
  for (int t = 0; t < T; ++t) {
    merged_count[t] = out_counts[0][(size_t)t];
    off[t + 1] = off[t] + (int64_t)out_sets[0][(size_t)t].size();
    if (sorted) std::copy(out_sets[0][(size_t)t].begin(), out_sets[0][(size_t)t].end(), sorted + off[t]);
  }
  return 0;
}

// Every rank calls the reference's MPI wrapper with its own demand row; remap[p*T + t] is
// what rank p holds after the broadcast.
int ref_hsdma_mpi(int P, int T, const int32_t *demand, const int32_t *node_of_gpu, int tasks_per_gpu,
                  int32_t *remap) {
  std::vector<GpuInfo> topo;
  std::vector<int> nodes(node_of_gpu, node_of_gpu + P);
  for (int g = 0; g < P; ++g) topo.push_back({g, node_of_gpu[g]});
  const int num_nodes = *std::max_element(nodes.begin(), nodes.end()) + 1;
  std::vector<int> status((size_t)P, 0);
  dsp_mpi_stub::run_ranks(P, [&](int p) {
    std::vector<int> mine(demand + (size_t)p * T, demand + (size_t)(p + 1) * T);
    std::vector<int> out((size_t)T, -1);
    ComputeAllocation_HSDMA_MPI(mine, topo, num_nodes, tasks_per_gpu, out, MPI_COMM_WORLD, 0, false);
    std::copy(out.begin(), out.end(), remap + (size_t)p * T);
  });
  return 0;
}
}
