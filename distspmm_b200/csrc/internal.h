// internal.h — host-side helpers shared by the library's translation units.
#pragma once
#include <stdarg.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "../../include/distspmm.h"
#include "common.h"

namespace dsp {

// Record a failure for dsp_last_error() on this thread and return `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

// Host worker count: DSP_HOST_THREADS if set, else hardware concurrency.
int host_threads();

// Run fn(begin, end) over [0, n) split into contiguous chunks on host threads.
void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)> &fn,
                  int64_t min_chunk = 4096);

// Work items of one CSR operand for the SpMM kernels (built on the host).
//   item_ptr[i] .. item_ptr[i+1]   nonzero range of item i (monotone, covers [0, nnz))
//   item_out[i] >= 0               output row of a whole-row item
//   item_out[i] <  0               piece of a split row; partial slot = -(item_out[i] + 1)
//   split_row[s], split_ptr[s..s+1] a split row and its consecutive partial slots
struct ItemPlan {
  std::vector<int64_t> item_ptr;
  std::vector<int32_t> item_out;
  std::vector<int32_t> split_row;
  std::vector<int32_t> split_ptr;
  int64_t piece_cap = 0;
  int64_t max_row_len = 0;
  int64_t pieces = 0;
};

// Piece length for a dense width: keeps the work of one piece near 32K multiply-adds.
int64_t default_piece_cap(int dims);

// Cut rows into items. rows: the output row of each listed row (nullptr = identity 0..m-1);
// row_ptr[m+1] nonzero ranges. include_empty: emit items for rows without nonzeros (so a
// non-accumulating launch writes their zeros).
void build_items(int64_t m, const int32_t *rows, const int64_t *row_ptr, int64_t piece_cap,
                 bool include_empty, ItemPlan *out);

// Equal nonzero chunks for the nnz-split kernels:
//   coo_row[p]           output row of nonzero p
//   chunk_slot[2c+0/1]   partial slot of chunk c's first / last row when that row crosses a
//                        chunk boundary, -1 when the chunk holds the whole row
//   split_row/split_ptr  rows crossing boundaries and their consecutive slots (chunk order)
struct ChunkPlan {
  std::vector<int32_t> coo_row;
  std::vector<int32_t> chunk_slot;
  std::vector<int32_t> split_row;
  std::vector<int32_t> split_ptr;
  int64_t chunk_nnz = 0;
  int64_t n_chunks = 0;
  int64_t slots = 0;
  int64_t max_row_len = 0;
};

// Nonzeros per chunk for a dense width (about 32K multiply-adds per chunk, fewer when the
// matrix is too small to give every SM enough chunks).
int64_t default_chunk_nnz(int dims, int64_t nnz);

void build_chunks(int64_t m, const int32_t *rows, const int64_t *row_ptr, int64_t chunk_nnz, ChunkPlan *out);

// Row-length statistics -> kRowSplit (0) for short, regular rows, kNnzSplit (1) otherwise.
int choose_variant(int64_t m, const int64_t *row_ptr, int dims);

}  // namespace dsp

#define DSP_TRY_ARG(cond, ...)                          \
  do {                                                  \
    if (!(cond)) return dsp::fail(DSP_ERR_INVALID, __VA_ARGS__); \
  } while (0)
