/*
 * distspmm.h — C ABI of the B200-native distributed CSR x dense SpMM engine.
 *
 * This is the drop-in boundary for the hot path of echogujy/DistSpMM:
 *   C[m x N] = A[m x M] (CSR, fp32 values, int64 indptr/indices) * B[M x N] (fp32, row-major)
 * with A split 1-D by rows over P ranks and B split into T = P * n_rolls row tiles that
 * are owned by ranks (slice / random / HSDMA allocation) and fetched bulk or
 * sparsity-aware over NVLink.
 *
 * The reference has no C ABI: its surface is header-only C++ plus the dist_spmm_node
 * CLI. Every entry point below cites the reference function (path:line, relative to
 * the reference repository) whose behaviour it reproduces or replaces.
 *
 * Conventions
 *   - Every function returns an int status: DSP_OK (0) or a negative DSP_ERR_* code.
 *     No exception and no exit() crosses this boundary. dsp_last_error() returns a
 *     thread-local message describing the last failure on the calling thread.
 *   - Output buffers are caller-owned unless the function allocates (dsp_csr_*,
 *     *_create), in which case a matching free/destroy function exists.
 *   - Streams are passed as void* (a cudaStream_t); NULL means the legacy default stream.
 *   - Objects are not thread-safe; drive one dsp_rank / dsp_spmm_plan from one host
 *     thread at a time.
 */
#ifndef DISTSPMM_H
#define DISTSPMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define DSP_OK 0
#define DSP_ERR_INVALID -1     /* bad argument (null pointer, out-of-range size)          */
#define DSP_ERR_IO -2          /* file missing, unreadable or shorter than declared        */
#define DSP_ERR_FORMAT -3      /* corrupt CSR: indptr not monotone / column out of range   */
#define DSP_ERR_CUDA -4        /* a CUDA runtime call failed                                */
#define DSP_ERR_NOMEM -5       /* host or device allocation failed                          */
#define DSP_ERR_UNSUPPORTED -6 /* valid input outside what this build handles              */
#define DSP_ERR_TIMEOUT -7     /* a bounded wait gave up                                    */
#define DSP_ERR_STATE -8       /* call out of order (e.g. peer buffer not attached)         */

const char *dsp_last_error(void);
const char *dsp_version(void);
/* Number of visible CUDA devices (0 on a host without a GPU; never fails). */
int dsp_device_count(void);

/* ---------------------------------------------------------------- host CSR */
/* Global or local CSR matrix in host memory, the reference's SparseMatrix<int64_t,float>
 * (src/sparse_matrix.h:19-65). Arrays allocated by the library are released by
 * dsp_csr_free(). */
typedef struct dsp_csr {
  int64_t num_rows;
  int64_t num_cols;
  int64_t nnz;
  int64_t *indptr;  /* num_rows + 1 */
  int64_t *indices; /* nnz, column ids */
  float *values;    /* nnz */
} dsp_csr;

/* Read <prefix>_indptr.bin (int64[M+1]), <prefix>_indices.bin (int64[nnz]) and
 * <prefix>_values.bin (fp32[nnz]); num_rows = filesize/8 - 1, nnz = indptr[M],
 * num_cols = num_rows (square). Replaces SparseMatrix::load_from_csr
 * (src/sparse_matrix.h:83-159). Same result on every well-formed file; unlike the
 * reference it returns DSP_ERR_IO on short files and DSP_ERR_FORMAT on a non-monotone
 * indptr or a column outside [0, num_cols) instead of reading garbage. Files longer than
 * declared are accepted and read up to nnz, as the reference does. A prefix ending in
 * ".mtx" returns DSP_ERR_UNSUPPORTED (the reference's load_from_mtx stub,
 * src/sparse_matrix.h:68-81, also refuses it). */
int dsp_csr_load(const char *prefix, dsp_csr *out);

/* Read only rows [row_lb, row_ub) of the binary CSR at <prefix> by seeking into the
 * three files; column ids stay global and indptr is rebased to 0. Equivalent to
 * load_from_csr followed by turn_local_l_u_csr (src/sparse_matrix.h:83-159, 178-199)
 * without every rank reading the whole matrix. num_cols is the global row count. */
int dsp_csr_load_rows(const char *prefix, int64_t row_lb, int64_t row_ub, dsp_csr *out);

/* Row count M of the binary CSR at <prefix> (from the size of <prefix>_indptr.bin) and, when
 * indptr is not NULL, the whole indptr[M+1]: what a rank needs to find its rows before it
 * reads them with dsp_csr_load_rows (src/sparse_matrix.h:85-101 reads the same file). */
int dsp_csr_read_indptr(const char *prefix, int64_t *M, int64_t *indptr);

/* Write the three binary files in the layout of tools/gen_graph500_matrix.py:40-49. */
int dsp_csr_save(const char *prefix, const dsp_csr *a);

/* Allocate an uninitialised CSR of the given shape (indptr zero-filled). */
int dsp_csr_alloc(int64_t num_rows, int64_t num_cols, int64_t nnz, dsp_csr *out);
void dsp_csr_free(dsp_csr *a);

/* Check indptr[0]==0, monotone indptr, indptr[M]==nnz and 0 <= col < num_cols. */
int dsp_csr_validate(const dsp_csr *a);

/* ---------------------------------------------------------------- synthetic inputs */
/* R-MAT (Chakrabarti et al.) with quadrant probabilities a, b, c (d = 1-a-b-c),
 * edge_factor * 2^scale edges, symmetrised, self-loops and duplicates removed, columns
 * ascending within a row, values U(0,1). Stands in for tools/gen_graph500_matrix.py:31-37
 * (NetworKit RmatGenerator, not available here). Deterministic in seed. */
int dsp_gen_rmat(int scale, int edge_factor, double a, double b, double c, uint64_t seed,
                 dsp_csr *out);
/* 27-point stencil on an n^3 grid, lexicographic ordering, diagonal 26.0, off-diagonals
 * U(-1,0). */
int dsp_gen_stencil27(int64_t n, uint64_t seed, dsp_csr *out);
/* Erdos-Renyi style: rows x rows, exactly nnz_per_row distinct uniform columns per row
 * (ascending), values U(0,1). */
int dsp_gen_uniform(int64_t rows, int64_t nnz_per_row, uint64_t seed, dsp_csr *out);
/* Dense rows [row0, row0+rows) of the synthetic B: element (r, c) = U(-1,1) from a
 * counter hash of (seed, r, c), identical on host and device. ld >= ncols. */
int dsp_fill_dense_host(float *B, int64_t row0, int64_t rows, int64_t ld, int64_t ncols,
                        uint64_t seed);
/* The same values for the listed global rows: B[i] = row rows[i] of the synthetic B (the
 * rows a sampled check needs, without materialising all of B). */
int dsp_fill_dense_rows_host(float *B, const int64_t *rows, int64_t n, int64_t ld, int64_t ncols,
                             uint64_t seed);

/* ---------------------------------------------------------------- planning (host, integer) */
/* 1-D row partition: m_local = ceil(M/P), lb = rank*m_local, ub = min(lb+m_local, M)
 * (src/dist_spmm_node.cu:85-91). lb may exceed M for trailing ranks; then ub = lb = M is
 * returned (the reference would produce a negative m_local there). */
int dsp_partition_bounds(int64_t M, int P, int rank, int64_t *lb, int64_t *ub);

/* Work-balanced 1-D row partition (no counterpart in the reference, whose equal-row split
 * gives rank 0 of an R-MAT graph ~40 % of the nonzeros): contiguous ranges [lb, ub) with
 * equal cost, cost = nonzeros + rows, i.e. rank p starts at the first row i where
 * indptr[i] - indptr[0] + i >= ceil(p * (nnz + M) / P). The ranges tile [0, M) in rank
 * order (a rank may be empty). indptr holds M + 1 entries. */
int dsp_partition_bounds_balanced(const int64_t *indptr, int64_t M, int P, int rank, int64_t *lb,
                                  int64_t *ub);

/* Local CSR of rows [lb, ub), indptr rebased, global column ids
 * (SparseMatrix::turn_local_l_u_csr, src/sparse_matrix.h:178-199). out->num_cols =
 * g->num_cols. */
int dsp_partition(const dsp_csr *g, int64_t lb, int64_t ub, dsp_csr *local);

/* Column tiling of a local CSR into T tiles of cpt = ceil(num_cols/T) columns
 * (src/dist_spmm_node.cu:103-132 and :210-223):
 *   cpt            -> *cpt_out
 *   n_col_list[t]  = number of distinct col % cpt in tile t (pre-merge, HSDMA demand)
 *   n_slice_list[t]= min(cpt, num_cols - t*cpt) if the tile holds a local nonzero, else 0
 *   nnz_list[t]    = number of local nonzeros in tile t
 * Any of the three output arrays may be NULL. */
int dsp_tile_counts(const dsp_csr *local, int T, int64_t *cpt_out, int32_t *n_col_list,
                    int32_t *n_slice_list, int64_t *nnz_list);

/* The per-tile needed column sets of the same tiling as ascending tile-local ids, flat:
 * tile t occupies cols[offsets[t] .. offsets[t+1]), offsets[t+1]-offsets[t] =
 * n_col_list[t]. The reference keeps them in std::unordered_set iteration order
 * (src/dist_spmm_node.cu:115-129); the set contents are identical. offsets has T+1
 * entries and is written by this call; cols must hold sum(n_col_list) ints. */
int dsp_tile_needed(const dsp_csr *local, int T, int64_t *offsets, int32_t *cols);

/* The same tiling on the current GPU, replacing the reference's per-nonzero unordered_set
 * loop (src/dist_spmm_node.cu:103-132). dsp_col_presence: d_present[c] = 1 for every column
 * c of the nnz device column ids d_cols (int64, the reference's index type), 0 elsewhere
 * (num_cols bytes, device); DSP_ERR_FORMAT if an id lies outside [0, num_cols).
 * Synchronous on `stream`. */
int dsp_col_presence(const int64_t *d_cols, int64_t nnz, int64_t num_cols, uint8_t *d_present,
                     void *stream);
/* Counts and ascending needed lists of dsp_tile_counts / dsp_tile_needed from device data:
 * n_col_list and the lists from d_present (computed from d_cols when NULL), n_slice_list and
 * nnz_list from d_cols (NULL with nnz = 0: no nonzeros, all zero). Node merge: pass the
 * element-wise maximum of the ranks' presence maps (an all-reduce, e.g. NCCL MAX on
 * uint8) as d_present and get the union lists of dsp_merge_needed. Outputs are host arrays
 * (any may be NULL; cols needs offsets and holds offsets[T] ids). T <= 8192. Synchronous. */
int dsp_tile_device(const int64_t *d_cols, int64_t nnz, const uint8_t *d_present, int64_t num_cols,
                    int T, int64_t *cpt_out, int32_t *n_col_list, int32_t *n_slice_list,
                    int64_t *nnz_list, int64_t *offsets, int32_t *cols, void *stream);

/* HSDMA two-phase greedy swap refinement (hierarchical_iterative_refinement_allocation,
 * src/h_sdma.h:78-228). demand is the P x T row-major matrix of pre-merge n_col_list
 * rows (rank-major), node_of_gpu[P] the node id of each rank (ranks of a node
 * contiguous). Writes remap[T] = owner rank of each tile, bit-identical to the reference
 * (strict-greater first maximum in lexicographic (a,b) order, exact integer costs). */
int dsp_hsdma(const int32_t *demand, int P, int T, const int32_t *node_of_gpu,
              int tasks_per_gpu, int max_inter_iters, int max_intra_iters, int32_t *remap);

/* task_dist 0: remap[t] = t / n_rolls (src/dist_spmm_node.cu:140-145). */
int dsp_alloc_slice(int P, int n_rolls, int32_t *remap);
/* task_dist 1: the reference shuffles iota(T) with the unseeded std::random_shuffle
 * (src/dist_spmm_node.cu:146-149), which yields owner ids >= P whenever n_rolls > 1.
 * Here: a seeded Fisher-Yates shuffle of the slice map, so every rank still owns n_rolls
 * tiles. Intentionally not bit-compatible. */
int dsp_alloc_random(int P, int n_rolls, uint64_t seed, int32_t *remap);

/* Node-level union of the needed sets (double_level_comm_node_processing,
 * src/utils.h:439-547). R ranks' sets, as their Allgather/Allgatherv would deliver them:
 * counts[R*T] (rank-major) and cols = rank 0's tiles 0..T-1, then rank 1's, ... Writes
 * n_col_merged[t] = |union_t| and merged_offsets[T+1]; if merged_cols is non-NULL it
 * receives the ascending union lists (size merged_offsets[T]). Call once with
 * merged_cols = NULL to size the buffer. */
int dsp_merge_needed(int R, int T, const int32_t *counts, const int32_t *cols,
                     int64_t *merged_offsets, int32_t *merged_cols, int32_t *n_col_merged);

/* Adaptive-communication model 1/(a*k^u + b/k), k = min(c, dims). */
typedef struct dsp_comm_model {
  float a, b, c, u;
} dsp_comm_model;

#define DSP_PLATFORM_H100 0 /* default of the reference (src/comm_man.h:391-394) */
#define DSP_PLATFORM_A800 1 /* DISTSPMM_PLATFORM_A800 (src/comm_man.h:387-390)    */
#define DSP_PLATFORM_B200 2 /* intra: fit of dsp_comm_probe on B200 NVLink 5     */
                            /* (a, b, c, u = 0.03045, 100.87679, 130.98926, 0.49); */
                            /* inter: H100's (no second node to measure)          */
#define DSP_TIER_INTRA 0
#define DSP_TIER_INTER 1
int dsp_comm_model_preset(int platform, int tier, dsp_comm_model *out);

/* Per-tile bulk/sparse decision (CommMan_hp::initialize_comm_model,
 * src/comm_man.h:369-410): comm_type 0 -> all bulk, 1 -> all sparse, 2 -> sparse iff
 * thr > n_col[i]/(n_slice[i]+1), evaluated in float with powf exactly as the reference.
 * sparse_inter may be NULL. */
int dsp_comm_select(int comm_type, int dims, const dsp_comm_model *intra,
                    const dsp_comm_model *inter, int T, const int32_t *n_col,
                    const int32_t *n_slice, uint8_t *sparse_intra, uint8_t *sparse_inter);

/* Communication traffic formulas (CommMan_hp::get_comm_traffic_intra / _inter,
 * src/comm_man.h:508-542), in bytes, for rank `me`. Inter-node traffic is 0 on one node;
 * dsp_traffic_inter implements the multi-node formula for ranks_per_node-sized nodes. */
int dsp_traffic_intra(int me, int T, const int32_t *remap, const uint8_t *sparse,
                      const int32_t *n_col, const int32_t *n_slice, int dims, int64_t *bytes);
int dsp_traffic_inter(int me, int ranks_per_node, int num_nodes, int T, const int32_t *remap,
                      const uint8_t *sparse_inter, const int32_t *n_col,
                      const int32_t *n_slice, int dims, int64_t *bytes);

/* 2 * nnz * dims / avg_ms / 1e6 (src/dist_spmm_node.cu:435). */
double dsp_gflops(int64_t nnz, int dims, double avg_ms);

/* ---------------------------------------------------------------- single-GPU SpMM */
/* A device-resident CSR operand prepared for the sm_100a SpMM kernels, column ids stored
 * as int32, cut into work units by one of two decompositions chosen from the row-length
 * statistics: row-split (one item per row, heavy rows cut into bounded pieces) or
 * nnz-split (equal chunks of consecutive nonzeros across row boundaries, with a row id
 * per nonzero). Partial rows are combined in a fixed order. Replaces the per-tile
 * cusparseCreateCoo + cusparseSpMM(ALG_DEFAULT) of src/dist_spmm_node.cu:233-234 and
 * :354-385. */
typedef struct dsp_spmm_plan dsp_spmm_plan;

typedef struct dsp_spmm_info {
  int64_t rows, cols, nnz;
  int64_t variant;     /* 0 = row-split items, 1 = nnz-split chunks     */
  int64_t items;       /* work units (row items or nonzero chunks)      */
  int64_t split_rows;  /* rows cut across work units                    */
  int64_t pieces;      /* partial-row scratch slots                     */
  int64_t piece_cap;   /* maximum nonzeros per unit                     */
  int64_t max_row_len; /* longest row                                   */
  int64_t scratch_bytes;
  int64_t device_bytes; /* all device memory the plan holds             */
} dsp_spmm_info;

/* Build the plan on `device` from a host CSR (indices < 2^31 required). dims_hint is the
 * dense width the plan is tuned for (it sets the piece / chunk length); variant: -1 picks
 * from the row-length statistics, 0 forces row-split, 1 forces nnz-split. */
#define DSP_VARIANT_AUTO -1
#define DSP_VARIANT_ROWS 0
#define DSP_VARIANT_NNZ 1
int dsp_spmm_plan_create(int device, const dsp_csr *a, int dims_hint, int variant, dsp_spmm_plan **out);
void dsp_spmm_plan_destroy(dsp_spmm_plan *p);
int dsp_spmm_plan_info(const dsp_spmm_plan *p, dsp_spmm_info *info);

/* C = A*B (accumulate = 0) or C += A*B (accumulate = 1), fp32 in and out, fp32
 * accumulation. B: cols x N device row-major with leading dimension ldb; C: rows x N,
 * ldc. Enqueued on `stream`; returns immediately. */
int dsp_spmm_f32(dsp_spmm_plan *p, const float *B, int64_t ldb, float *C, int64_t ldc, int N,
                 int accumulate, void *stream);
/* After the stream of earlier dsp_spmm_f32 calls was synchronised: DSP_OK, or
 * DSP_ERR_TIMEOUT if a kernel's bounded wait on its shared-memory copies gave up (the
 * banded kernel's staged windows); the flag is cleared. Not in the reference (no failure
 * detection there, src/utils.h:26-84). */
int dsp_spmm_check_error(dsp_spmm_plan *p);

/* Allocation-free SpMM (no counterpart in the reference). C = A*B (accumulate = 0) or
 * C += A*B on the current CUDA device, for a CSR matrix the caller already holds in device
 * memory in the reference's layout (int64 indptr[rows+1], int64 indices[nnz], fp32
 * values[nnz]); B (cols x N, ldb) and C (rows x N, ldc) as for dsp_spmm_f32.
 * For callers that cannot call cudaMalloc: code on a latency-critical stream beside other
 * work (cudaMalloc / cudaFree may synchronise the device), frameworks whose own memory pool
 * owns the device and forbids allocations behind its back, and steps that must not fail
 * with out-of-memory midway. It allocates no device memory and calls no allocating
 * routine: its only scratch (partial rows of rows cut between work chunks) is a static
 * 32 MiB device array that every GPU loading the library holds until exit.
 * Limits: N <= DSP_NOALLOC_MAX_N and rows < 2^31 (DSP_ERR_UNSUPPORTED otherwise).
 * Set-up: the first call on a device looks up that device's scratch address
 * (cudaGetSymbolAddress, once per device, cached for the process). Under lazy module
 * loading that first lookup may also load the library's device code together with its
 * 32 MiB array, which allocates and can synchronise the device. So make one call per device
 * before any stream capture or latency-critical work; a call with N = 0 or rows = 0 does the
 * set-up and touches no memory. The cached address belongs to the device's context
 * at that time: do not use this entry point on a device after cudaDeviceReset.
 * All calls on a device share the scratch: calls that overlap on the GPU (e.g. on two
 * streams) race; serialise them. The scratch keeps the last call's contents; no call relies
 * on it being zero. */
#define DSP_NOALLOC_MAX_N 2048
int dsp_spmm_csr_f32_noalloc(const int64_t *indptr, const int64_t *indices, const float *values,
                             int64_t rows, int64_t cols, int64_t nnz, const float *B, int64_t ldb,
                             float *C, int64_t ldc, int N, int accumulate, void *stream);

/* ---------------------------------------------------------------- distributed rank */
/* One GPU's share of the distributed SpMM: the local rows of A cut into segments by the
 * owner of each column tile (own tiles first, then peers in ring order (me+k)%P as in
 * src/dist_spmm_node.cu:339-343), a full-height B buffer in which the owned tiles live at
 * their global row offsets and fetched remote rows land at the same offsets, and C. */
typedef struct dsp_rank dsp_rank;

typedef struct dsp_rank_desc {
  int rank;             /* this rank, 0 <= rank < world                         */
  int world;            /* P                                                     */
  int device;           /* CUDA device ordinal                                  */
  int dims;             /* N, dense width                                       */
  int T;                /* total tiles = P * n_rolls                            */
  int n_streams;        /* concurrent fetch streams (nvlink_num_producers)      */
  int64_t cpt;          /* rows per tile, ceil(M/T)                             */
  int64_t M;            /* global rows = global columns                         */
  int64_t m_lb;         /* first global row of this rank                        */
  const dsp_csr *local; /* local rows, global column ids                        */
  const int32_t *remap;          /* [T] owner rank of each tile                 */
  const uint8_t *sparse;         /* [T] 1 = sparsity-aware fetch, 0 = bulk      */
  const int64_t *needed_offsets; /* [T+1] merged needed lists                   */
  const int32_t *needed_cols;    /* tile-local ids, ascending per tile          */
  const int32_t *n_slice;        /* [T] n_slice_list of this rank               */
  int fetch_engine;              /* DSP_FETCH_LSU (default) or DSP_FETCH_TMA     */
  int pipeline;                  /* DSP_PIPELINE_* (0 = pick from the matrix)    */
  int groups;                    /* DSP_PIPELINE_GROUPS: row groups (0 = 8)      */
} dsp_rank_desc;

/* How a rank's nonzeros are cut into phases, phase k running once the fetches of ring
 * positions 1..k (peer (rank + k) % P) have landed:
 *   ROWS   whole rows, in the phase of the last ring position their columns need: every C
 *          row written once (no read-modify-write); best when most rows need only owned
 *          tiles (banded / mesh matrices).
 *   SPLIT  nonzeros by the ring position owning their column, as the reference's per-tile
 *          loop (src/dist_spmm_node.cu:329-394): a row is written in its first phase and
 *          accumulated in later ones, so compute overlaps every fetch; best when nearly all
 *          rows need remote tiles (power-law graphs).
 *   GROUPS (no counterpart in the reference) first the nonzeros of every row whose tiles
 *          this rank owns (no fetch needed), then the local rows in `groups` contiguous
 *          groups of equal work, each group's remote nonzeros added to those rows: every
 *          remote row is fetched with the first group that needs it, from every peer at
 *          once, and group g runs once the fetches of groups 0..g have landed, so the
 *          fetches hide behind the owned-column pass and earlier groups' SpMM; a row is
 *          written once and read back at most once. Each rank fetches only the rows its own
 *          nonzeros need (the node-merged lists are not used). For power-law graphs, whose
 *          rows need every peer: at P = 8 the first of 8 groups needs ~40 % of a rank's
 *          remote rows and each later group 5-16 %.
 *   AUTO   ROWS when at least half the nonzeros fall in its phase 0; otherwise SPLIT when
 *          the owned tiles hold enough work and the accumulated pieces are long, else
 *          GROUPS. */
#define DSP_PIPELINE_AUTO 0
#define DSP_PIPELINE_ROWS 1
#define DSP_PIPELINE_SPLIT 2
#define DSP_PIPELINE_GROUPS 3

/* Sparse-fetch engines: LSU = warps with 128-bit peer loads, one block per SM next to the
 * SpMM; TMA = per-row cp.async.bulk copies through a shared-memory ring (no multicast). */
#define DSP_FETCH_LSU 0
#define DSP_FETCH_TMA 1

typedef struct dsp_rank_stats {
  int64_t m_local, nnz_local;
  int64_t segments;          /* owners this rank computes against (incl. itself) */
  int64_t fetch_rows;        /* remote B rows moved per step                     */
  int64_t fetch_bytes;       /* remote bytes moved per step                      */
  int64_t fetch_bulk_tiles;  /* tiles fetched whole                              */
  int64_t fetch_sparse_tiles;/* tiles fetched row by row                         */
  int64_t owned_rows;        /* B rows this rank owns                            */
  int64_t distinct_cols;     /* distinct columns of the local rows (U_p)         */
  int64_t launches_per_step; /* kernels + copies enqueued per step               */
  int64_t kernels_per_step;  /* of which kernels of this library                  */
  int64_t device_bytes;      /* device memory held by the rank                   */
  int64_t pipeline;          /* DSP_PIPELINE_ROWS, _SPLIT or _GROUPS in use      */
  int64_t phase0_nnz;        /* nonzeros computed before any fetch lands         */
  int64_t timeline_len;      /* entries of dsp_rank_last_timeline (max(P, groups)) */
  /* DSP_PIPELINE_AUTO's step-time model of the three phase structures for this rank (ms) */
  float model_rows_ms, model_split_ms, model_groups_ms;
} dsp_rank_stats;

int dsp_rank_create(const dsp_rank_desc *d, dsp_rank **out);
void dsp_rank_destroy(dsp_rank *r);
int dsp_rank_stats_get(const dsp_rank *r, dsp_rank_stats *s);
int dsp_rank_b_ptr(dsp_rank *r, float **B);
int dsp_rank_c_ptr(dsp_rank *r, float **C);
/* CUDA IPC handle (64 bytes) of this rank's B buffer, for peers in other processes. */
int dsp_rank_ipc_handle(dsp_rank *r, void *handle64);
/* Attach a peer's B buffer: from an IPC handle (other process) or a pointer that is
 * valid on this rank's device (same process; peer access is enabled when needed). */
int dsp_rank_open_peer(dsp_rank *r, int peer, const void *handle64);
int dsp_rank_set_peer(dsp_rank *r, int peer, const float *peer_B, int peer_device);
/* Fill the owned tiles of B with the synthetic U(-1,1) values (dsp_fill_dense_host). */
int dsp_rank_fill_b(dsp_rank *r, uint64_t seed, void *stream);
/* Debug aid: fill every B row this rank does not own with NaN, so that a remote row a
 * step failed to fetch (or fetched late) poisons C instead of passing silently. */
int dsp_rank_poison_remote(dsp_rank *r, void *stream);
/* Copy the owned tiles of a full host B (M x dims, row-major) into the device B. */
int dsp_rank_upload_b(dsp_rank *r, const float *B_host, void *stream);
/* Same from a host buffer holding only the owned tiles, back to back in ascending tile
 * order (owned_rows x dims, dsp_rank_stats.owned_rows): a rank's share of B without a full
 * M x dims host copy. */
int dsp_rank_upload_b_owned(dsp_rank *r, const float *B_owned_host, void *stream);
/* One distributed SpMM: fetch the needed remote rows (bulk copy-engine copies and
 * sparse NVLink gather kernels on the fetch streams) while the SpMM kernels run segment
 * by segment on the compute stream; C = A_local * B. Ordered after prior work on
 * `stream`; later work on `stream` is ordered after it. Peers' owned tiles must hold the
 * step's B before the call (the caller's barrier). */
int dsp_rank_step(dsp_rank *r, void *stream);
/* After the step's stream was synchronised: DSP_OK, or DSP_ERR_TIMEOUT if a fetch kernel's
 * or the banded SpMM kernel's bounded wait on its bulk copies gave up during an earlier
 * step (the flag is cleared).
 * The reference has no failure detection (src/utils.h:26-84 exit() on any error). */
int dsp_rank_check_error(dsp_rank *r);
/* Test of the fetch kernels' bounded wait on the current device: one CTA waits on an
 * mbarrier that nothing arrives at, for budget_cycles clock64 cycles (<= ~2 s), then
 * records code 3 and returns. Returns DSP_ERR_TIMEOUT with *code_out = 3 when the wait gave
 * up as designed, DSP_OK if it (impossibly) completed. No fault, no hang. */
int dsp_selftest_bounded_wait(long long budget_cycles, int *code_out);
/* Bulk-vs-sparse fetch microbenchmark, the reference's comm_test (src/comm_test.cu:83-147)
 * on this engine's fetch paths: *bulk_ms = one copy-engine copy of peer_device's whole
 * rows x dims fp32 buffer into device; sparse_ms[i] = the gather kernel of `engine`
 * (DSP_FETCH_*) moving the first counts[i] rows of row_ids (host, < rows) the same way.
 * Mean of `reps` timed launches (CUDA events) after one untimed launch; the buffers are
 * allocated and freed by the call. peer_device == device measures a local copy. */
int dsp_comm_probe(int device, int peer_device, int64_t rows, int dims, const int32_t *row_ids,
                   int n_counts, const int64_t *counts, int engine, int reps, double *bulk_ms,
                   double *sparse_ms);
/* Copy C (m_local x dims) to host. */
int dsp_rank_download_c(dsp_rank *r, float *C_host, void *stream);
/* Device time (ms) of the SpMM kernels of the last step, from CUDA events on the compute
 * stream (valid after the step completed). */
int dsp_rank_last_compute_ms(dsp_rank *r, float *ms);
/* Timeline of the last step (valid after it completed), ms from the step's start, 4 floats
 * per entry k < dsp_rank_stats.timeline_len: fetch begin, fetch end of ring position k (peer
 * (me+k)%P, k < P), segment begin, segment end of phase (or row group) k; -1 where nothing
 * ran. cap >= 4 * timeline_len. Shows how much of the fetch the SpMM segments hid (the
 * reference measures only whole reps, src/dist_spmm_node.cu:329-394). */
int dsp_rank_last_timeline(dsp_rank *r, float *ms, int cap);

/* ---------------------------------------------------------------- whole pipeline */
/* The dist_spmm_node program (src/dist_spmm_node.cu:20-444) run in one process that
 * drives `world` ranks (one host thread each) on devices[rank] (ranks may share a GPU).
 * Host collectives that the reference does with MPI happen in shared memory. */
typedef struct dsp_args {
  const char *file;   /* CSR prefix, or NULL to use `matrix`                  */
  const dsp_csr *matrix;
  int dims, task_dist, comm_type, n_rolls, repeat, n_streams;
  int world;
  const int *devices; /* [world]                                              */
  int platform;       /* DSP_PLATFORM_*                                       */
  uint64_t b_seed;    /* B = synthetic U(-1,1) (reference: all ones)          */
  int b_ones;         /* 1: B filled with 1.0 as the reference does           */
  float *c_out;       /* optional host [M x dims] to receive C                */
} dsp_args;

typedef struct dsp_report {
  double stage_ms[8];  /* read, partition, tiling, allocation, merge, device setup,
                          comm manager, streams (reference time_costs[0..7])   */
  double hsdma_ms;
  double avg_ms, min_ms, median_ms; /* per-rep wall time, max over ranks, reps >= 5 */
  int reps_counted;
  int64_t traffic_intra, traffic_inter; /* reference formula, summed over ranks */
  int64_t fetched_bytes;                /* bytes actually moved, summed          */
  double mem_gb;                        /* device memory held by the engine      */
  double gflops;
  int64_t nnz, M;
  int T;
  int32_t remap[4096];
  int64_t row_lb, row_ub;               /* dsp_run_rank: this rank's rows           */
} dsp_report;

int dsp_run(const dsp_args *args, dsp_report *report);

/* ---------------------------------------------------------------- one process per rank */
/* Host collectives for ranks launched as separate processes on one node, in place of the
 * reference's MPI (MPI_Gather/Bcast of src/utils.h:358-437, MPI_Allgather(v) of
 * src/utils.h:439-547, MPI_Allreduce of src/dist_spmm_node.cu:401-409). The ranks meet in a
 * directory every process of the job can reach (tmpfs); each value is one file written
 * atomically; every wait is bounded by timeout_s (<= 0: 300 s) and then fails with
 * DSP_ERR_TIMEOUT, so a rank that died or never started is reported instead of hanging
 * the others. Every rank makes the same calls with the same keys in the same order; a
 * key is used once per store. */
typedef struct dsp_store dsp_store;
int dsp_store_open(const char *dir, int rank, int world, double timeout_s, dsp_store **out);
/* Publish `bytes` bytes under key and collect every rank's value, rank by rank, into out
 * (capacity out_cap; NULL to collect sizes only); sizes[world] receives each rank's size
 * (may be NULL). */
int dsp_store_allgather(dsp_store *s, const char *key, const void *data, int64_t bytes, void *out,
                        int64_t out_cap, int64_t *sizes);
int dsp_store_barrier(dsp_store *s, const char *key);
/* remove_dir: after every rank's last collective, rank 0 deletes the directory (every
 * rank must close with the same flag). */
void dsp_store_close(dsp_store *s, int remove_dir);

/* Rank `rank` of `world` of the dist_spmm_node program (src/dist_spmm_node.cu:20-444) when
 * every rank is its own process on its own GPU (`device`), as under `mpirun -np P`
 * (src/utils.h:176-237 binds a rank to the GPU of its node-local rank). args->world and
 * args->devices are ignored; the rank reads only its own rows of args->file; peers' B
 * buffers are opened by CUDA IPC. Every rank gets the same report (times MAX over ranks,
 * traffic summed), plus its own row range; args->c_out, when set, receives this rank's
 * rows of C ([row_ub - row_lb] x dims). */
int dsp_run_rank(const dsp_args *args, int rank, int world, int device, dsp_store *store,
                 dsp_report *report);

#ifdef __cplusplus
}
#endif
#endif /* DISTSPMM_H */
