// device.cuh — device-side declarations shared by the CUDA translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.h"

namespace dsp {

constexpr int kSpmmThreads = 256;
// Diagonal (DIA) form of banded operands: at most kMaxDiag distinct offsets col - row,
// blocks of kDiaRows consecutive rows per warp (one presence byte per block and diagonal).
constexpr int kMaxDiag = 32;
constexpr int kDiaRows = 8;

// The two SpMM work decompositions (picked per operand from its row-length statistics).
enum SpmmVariant : int {
  kRowSplit = 0,  // one item per row (heavy rows cut into pieces): regular, short-tailed rows
  kNnzSplit = 1,  // equal nonzero chunks across row boundaries (merge-path style): skewed rows
};

// Arguments of one SpMM launch (passed by value to the kernels).
struct SpmmArgs {
  int variant;
  // row-split
  const int64_t *item_ptr;  // [n_items + 1]
  const int32_t *item_out;  // [n_items]  row (>= 0) or -(slot + 1)
  int64_t n_items;
  // nnz-split
  const int32_t *coo_row;     // [nnz] output row of each nonzero
  const int32_t *chunk_slot;  // [2 * n_chunks] partial slot of the head / tail row, -1 if whole
  int64_t n_chunks;
  int64_t chunk_nnz;
  int64_t nnz;
  int64_t zero_rows;  // rows [0, zero_rows) without nonzeros are written as 0 (non-accumulating)
  // both: rows cut across items / chunks, summed into C by the fixup kernel
  const int32_t *split_row;  // [n_split]
  const int32_t *split_ptr;  // [n_split + 1] slot ranges
  int64_t n_split;
  const int32_t *cols;  // [nnz]
  const float *vals;    // [nnz]
  const float *B;
  int64_t ldb;
  int64_t b_rows;  // rows of B (the operand's columns); 0 = unknown
  float *C;
  int64_t ldc;
  float *partial;  // [slots][N]
  int N;
  // split pipeline: output row r is accumulated (C += ...) when first_phase[r] < phase,
  // written otherwise; nullptr = every row written (or accumulated, per the launch)
  const uint8_t *first_phase;
  int phase;
  // row-split operands that are banded: the diagonal form (nullptr when the operand has none)
  const float *dia_vals;    // [n_diag][dia_m] value of (row i, col i + diag_off[d]), 0 if absent
  const uint8_t *dia_pres;  // [ceil(dia_m / kDiaRows)][n_diag] bit r: row 8b + r has that entry
  int64_t dia_m;            // listed rows (consecutive output rows from dia_row0)
  int64_t dia_row0;
  int n_diag;
  int32_t diag_off[kMaxDiag];   // ascending
  int n_runs;                    // runs of consecutive offsets (o, o+1, ..., at most 4 long)
  uint8_t run_len[kMaxDiag];     // in offset order
  int *err;  // device error word set by a kernel whose bounded wait gave up (nullptr: none)
  uint32_t wait_hint_ns;  // suspend-time hint of the staged kernels' mbarrier waits (0: none)
};

struct SpmmShape {
  int W;           // floats per vector (8, 4 or 1)
  int LPR;         // lanes per item / chunk
  int VPL;         // vectors per lane
  int chunk_cols;  // columns per blockIdx.y
  int chunks;
};

// max_w caps the vector width for kernels instantiated only up to float4.
SpmmShape spmm_shape(int N, int variant, const float *B, int64_t ldb, const float *C, int64_t ldc,
                     int max_w = 8);
int launch_spmm(const SpmmArgs &a, bool accumulate, cudaStream_t stream);
int launch_fill_dense(float *B, int64_t row0, int64_t rows, int64_t ld, int64_t ncols, uint64_t seed,
                      cudaStream_t stream);
int launch_fill_const(float *B, int64_t n, float v, cudaStream_t stream);
// dst[r, :] = src[r, :] for the global rows r = rows[0..n) (src: a peer's B). A wait that
// gives up sets *err (non-zero) instead of hanging.
int launch_gather_rows(float *dst, const float *src, const int32_t *rows, int64_t n, int dims, int engine, int *err,
                       cudaStream_t s);
// C[rows[i], 0:N] = 0 for i < n.
int launch_zero_rows(float *C, int64_t ldc, const int32_t *rows, int64_t n, int N, cudaStream_t stream);
void prefer_l1_carveout();
int dev_upload(void *dptr_out, const void *host, size_t bytes);

// A CSR operand in device memory, cut into work items (row-split) or nonzero chunks
// (nnz-split).
struct DevOperand {
  int device = 0;
  int variant = kRowSplit;
  int64_t rows = 0, cols = 0, nnz = 0;
  int64_t n_items = 0, n_chunks = 0, chunk_nnz = 0, n_split = 0, pieces = 0, piece_cap = 0, max_row_len = 0;
  int64_t zero_rows = 0;
  int64_t *d_item_ptr = nullptr;
  int32_t *d_item_out = nullptr;
  int32_t *d_coo_row = nullptr;
  int32_t *d_chunk_slot = nullptr;
  int64_t n_lrows = 0;   // rows the operand lists (the diagonal form's row count)
  int64_t hot_cols = 0;  // columns whose B rows are read with evict_last (mark_hot_columns)
  int32_t *d_split_row = nullptr;
  int32_t *d_split_ptr = nullptr;
  int32_t *d_cols = nullptr;
  float *d_vals = nullptr;
  // diagonal form (row-split operands whose listed rows are consecutive and that have at
  // most kMaxDiag distinct offsets, densely filled)
  float *d_dia_vals = nullptr;
  uint8_t *d_dia_pres = nullptr;
  int64_t dia_row0 = 0;
  int n_diag = 0;
  int32_t diag_off[kMaxDiag] = {};
  int n_runs = 0;
  uint8_t run_len[kMaxDiag] = {};

  // Rows i < m with nonzeros [row_ptr[i], row_ptr[i+1]) of indices/values (offsets are
  // absolute; first_nz is subtracted); row_ids[i] is the output row (nullptr = i).
  // include_empty: the operand writes every output row [0, rows) (non-accumulating use).
  // dims: the dense width it is tuned for; variant < 0 picks from the row statistics.
  int upload(int device, int64_t rows, int64_t cols, const int64_t *row_ptr, const int32_t *row_ids, int64_t m,
             const int64_t *indices, const float *values, int64_t first_nz, int64_t nnz, int dims,
             bool include_empty, int variant = -1);
  void release();
  // work units a launch covers: row items (row-split) or nonzero chunks (nnz-split)
  int64_t units() const { return variant == kRowSplit ? n_items : n_chunks; }
  int64_t device_bytes() const;
  SpmmArgs args(const float *B, int64_t ldb, float *C, int64_t ldc, int N, float *partial) const;
};

}  // namespace dsp
