// host_csr.cpp — error reporting, host threading, and the binary CSR format
// (load / partial load / save / validate / 1-D partition).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include <mutex>

#include "internal.h"

namespace dsp {

static thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int host_threads() {
  static int n = [] {
    const char *e = getenv("DSP_HOST_THREADS");
    int v = e ? atoi(e) : 0;
    if (v <= 0) v = (int)std::thread::hardware_concurrency();
    return v > 0 ? v : 1;
  }();
  return n;
}

void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)> &fn, int64_t min_chunk) {
  if (n <= 0) return;
  int64_t nt = std::min<int64_t>(host_threads(), (n + min_chunk - 1) / min_chunk);
  if (nt <= 1) {
    fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  th.reserve(nt);
  for (int64_t t = 0; t < nt; ++t) {
    int64_t b = n * t / nt, e = n * (t + 1) / nt;
    th.emplace_back([&fn, b, e] { fn(b, e); });
  }
  for (auto &x : th) x.join();
}

}  // namespace dsp

using namespace dsp;

extern "C" const char *dsp_last_error(void) { return g_last_error.c_str(); }
extern "C" const char *dsp_version(void) { return "distspmm_b200 0.1 (sm_100a)"; }

// ----------------------------------------------------------------- allocation

extern "C" int dsp_csr_alloc(int64_t num_rows, int64_t num_cols, int64_t nnz, dsp_csr *out) {
  DSP_TRY_ARG(out, "dsp_csr_alloc: out is NULL");
  DSP_TRY_ARG(num_rows >= 0 && num_cols >= 0 && nnz >= 0, "dsp_csr_alloc: negative size");
  memset(out, 0, sizeof *out);
  out->indptr = (int64_t *)calloc((size_t)num_rows + 1, sizeof(int64_t));
  out->indices = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nnz > 0 ? nnz : 1));
  out->values = (float *)malloc(sizeof(float) * (size_t)(nnz > 0 ? nnz : 1));
  if (!out->indptr || !out->indices || !out->values) {
    dsp_csr_free(out);
    return fail(DSP_ERR_NOMEM, "dsp_csr_alloc: out of host memory (%lld nnz)", (long long)nnz);
  }
  out->num_rows = num_rows;
  out->num_cols = num_cols;
  out->nnz = nnz;
  return DSP_OK;
}

extern "C" void dsp_csr_free(dsp_csr *a) {
  if (!a) return;
  free(a->indptr);
  free(a->indices);
  free(a->values);
  memset(a, 0, sizeof *a);
}

// ----------------------------------------------------------------- validation

extern "C" int dsp_csr_validate(const dsp_csr *a) {
  DSP_TRY_ARG(a && a->indptr, "dsp_csr_validate: null matrix");
  if (a->indptr[0] != 0) return fail(DSP_ERR_FORMAT, "indptr[0] = %lld, expected 0", (long long)a->indptr[0]);
  if (a->indptr[a->num_rows] != a->nnz)
    return fail(DSP_ERR_FORMAT, "indptr[M] = %lld but nnz = %lld", (long long)a->indptr[a->num_rows],
                (long long)a->nnz);
  std::atomic<int64_t> bad_row{-1}, bad_nz{-1};
  parallel_for(a->num_rows, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i)
      if (a->indptr[i + 1] < a->indptr[i]) {
        bad_row.store(i);
        return;
      }
  });
  if (bad_row.load() >= 0)
    return fail(DSP_ERR_FORMAT, "indptr not monotone at row %lld", (long long)bad_row.load());
  const int64_t nc = a->num_cols;
  parallel_for(a->nnz, [&](int64_t b, int64_t e) {
    for (int64_t j = b; j < e; ++j)
      if (a->indices[j] < 0 || a->indices[j] >= nc) {
        bad_nz.store(j);
        return;
      }
  });
  if (bad_nz.load() >= 0)
    return fail(DSP_ERR_FORMAT, "column %lld at nonzero %lld outside [0, %lld)",
                (long long)a->indices[bad_nz.load()], (long long)bad_nz.load(), (long long)nc);
  return DSP_OK;
}

// ----------------------------------------------------------------- file I/O

namespace {

struct File {
  FILE *f = nullptr;
  ~File() {
    if (f) fclose(f);
  }
};

int64_t file_size(const std::string &path) {
  struct stat st;
  if (stat(path.c_str(), &st) != 0) return -1;
  return (int64_t)st.st_size;
}

bool ends_with(const std::string &s, const char *suf) {
  size_t n = strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

// Read `count` elements of `size` bytes at element offset `first`.
int read_at(const std::string &path, int64_t first, int64_t count, size_t size, void *dst) {
  File f;
  f.f = fopen(path.c_str(), "rb");
  if (!f.f) return fail(DSP_ERR_IO, "cannot open %s", path.c_str());
  if (count == 0) return DSP_OK;
  if (fseeko(f.f, (off_t)(first * (int64_t)size), SEEK_SET) != 0)
    return fail(DSP_ERR_IO, "seek failed in %s", path.c_str());
  size_t got = fread(dst, size, (size_t)count, f.f);
  if ((int64_t)got != count)
    return fail(DSP_ERR_IO, "%s: short read (%lld of %lld elements from offset %lld)", path.c_str(),
                (long long)got, (long long)count, (long long)first);
  return DSP_OK;
}

int open_rows(const std::string &prefix, int64_t *M) {
  if (ends_with(prefix, ".mtx"))
    return fail(DSP_ERR_UNSUPPORTED, "%s: .mtx input is not implemented (the reference refuses it too)",
                prefix.c_str());
  std::string ip = prefix + "_indptr.bin";
  int64_t sz = file_size(ip);
  if (sz < 0) return fail(DSP_ERR_IO, "Failed to open row pointer file: %s", ip.c_str());
  if (sz < 8 || sz % 8 != 0)
    return fail(DSP_ERR_FORMAT, "%s: size %lld is not a positive multiple of 8", ip.c_str(), (long long)sz);
  *M = sz / 8 - 1;
  return DSP_OK;
}

}  // namespace

extern "C" int dsp_csr_load_rows(const char *prefix_c, int64_t row_lb, int64_t row_ub, dsp_csr *out) {
  DSP_TRY_ARG(prefix_c && out, "dsp_csr_load_rows: null argument");
  std::string prefix(prefix_c);
  int64_t M = 0;
  int rc = open_rows(prefix, &M);
  if (rc) return rc;
  DSP_TRY_ARG(row_lb >= 0 && row_lb <= row_ub && row_ub <= M,
              "dsp_csr_load_rows: rows [%lld, %lld) outside [0, %lld]", (long long)row_lb,
              (long long)row_ub, (long long)M);
  const int64_t m = row_ub - row_lb;
  std::vector<int64_t> ptr((size_t)m + 1);
  if ((rc = read_at(prefix + "_indptr.bin", row_lb, m + 1, 8, ptr.data()))) return rc;
  int64_t first = ptr[0], nnz = ptr[m] - ptr[0];
  if (row_lb == 0 && first != 0) return fail(DSP_ERR_FORMAT, "%s: indptr[0] = %lld", prefix_c, (long long)first);
  if (nnz < 0) return fail(DSP_ERR_FORMAT, "%s: indptr decreases", prefix_c);
  if ((rc = dsp_csr_alloc(m, M, nnz, out))) return rc;
  for (int64_t i = 0; i <= m; ++i) out->indptr[i] = ptr[i] - first;
  if ((rc = read_at(prefix + "_indices.bin", first, nnz, 8, out->indices)) ||
      (rc = read_at(prefix + "_values.bin", first, nnz, 4, out->values))) {
    dsp_csr_free(out);
    return rc;
  }
  if ((rc = dsp_csr_validate(out))) {
    std::string msg = std::string(prefix_c) + ": " + dsp_last_error();
    dsp_csr_free(out);
    return fail(rc, "%s", msg.c_str());
  }
  return DSP_OK;
}

extern "C" int dsp_csr_read_indptr(const char *prefix_c, int64_t *M, int64_t *indptr) {
  DSP_TRY_ARG(prefix_c && M, "dsp_csr_read_indptr: null argument");
  std::string prefix(prefix_c);
  int rc = open_rows(prefix, M);
  if (rc || !indptr) return rc;
  return read_at(prefix + "_indptr.bin", 0, *M + 1, 8, indptr);
}

extern "C" int dsp_csr_load(const char *prefix, dsp_csr *out) {
  DSP_TRY_ARG(prefix && out, "dsp_csr_load: null argument");
  int64_t M = 0;
  int rc = open_rows(prefix, &M);
  if (rc) return rc;
  return dsp_csr_load_rows(prefix, 0, M, out);
}

extern "C" int dsp_csr_save(const char *prefix_c, const dsp_csr *a) {
  DSP_TRY_ARG(prefix_c && a && a->indptr, "dsp_csr_save: null argument");
  std::string prefix(prefix_c);
  struct Part {
    const char *suffix;
    const void *data;
    size_t size;
    int64_t count;
  } parts[3] = {{"_indptr.bin", a->indptr, 8, a->num_rows + 1},
                {"_indices.bin", a->indices, 8, a->nnz},
                {"_values.bin", a->values, 4, a->nnz}};
  for (auto &p : parts) {
    std::string path = prefix + p.suffix;
    File f;
    f.f = fopen(path.c_str(), "wb");
    if (!f.f) return fail(DSP_ERR_IO, "cannot create %s", path.c_str());
    if (p.count && fwrite(p.data, p.size, (size_t)p.count, f.f) != (size_t)p.count)
      return fail(DSP_ERR_IO, "short write to %s", path.c_str());
  }
  return DSP_OK;
}

// ----------------------------------------------------------------- partition

extern "C" int dsp_partition_bounds(int64_t M, int P, int rank, int64_t *lb, int64_t *ub) {
  DSP_TRY_ARG(lb && ub && P > 0 && rank >= 0 && rank < P && M >= 0, "dsp_partition_bounds: bad argument");
  int64_t m_local = (M + P - 1) / P;
  int64_t l = (int64_t)rank * m_local;
  if (l > M) l = M;
  *lb = l;
  *ub = std::min(l + m_local, M);
  return DSP_OK;
}

// Contiguous rows with equal work: cost(rows [0, i)) = indptr[i] + i (one B-row gather per
// nonzero, one C-row write per row); rank p starts at the first row whose prefix cost
// reaches p/P of the total. Boundaries are monotone in p, so the P ranges tile [0, M).
extern "C" int dsp_partition_bounds_balanced(const int64_t *indptr, int64_t M, int P, int rank, int64_t *lb,
                                             int64_t *ub) {
  DSP_TRY_ARG(indptr && lb && ub && P > 0 && rank >= 0 && rank < P && M >= 0,
              "dsp_partition_bounds_balanced: bad argument");
  const int64_t total = indptr[M] - indptr[0] + M;
  auto start = [&](int p) -> int64_t {
    if (p <= 0) return 0;
    if (p >= P) return M;
    // target = ceil(total * p / P) without overflow for totals below 2^62 / P
    const int64_t target = (int64_t)(((__int128)total * p + P - 1) / P);
    int64_t lo = 0, hi = M;  // first i in [0, M] with cost(i) >= target
    while (lo < hi) {
      const int64_t mid = lo + (hi - lo) / 2;
      if (indptr[mid] - indptr[0] + mid >= target)
        hi = mid;
      else
        lo = mid + 1;
    }
    return lo;
  };
  *lb = start(rank);
  *ub = start(rank + 1);
  return DSP_OK;
}

extern "C" int dsp_partition(const dsp_csr *g, int64_t lb, int64_t ub, dsp_csr *local) {
  DSP_TRY_ARG(g && local && g->indptr, "dsp_partition: null argument");
  if (lb < 0 || ub > g->num_rows || lb > ub)
    return fail(DSP_ERR_INVALID, "Invalid partition range [%lld, %lld) of %lld rows", (long long)lb,
                (long long)ub, (long long)g->num_rows);
  const int64_t start = g->indptr[lb], end = g->indptr[ub], m = ub - lb;
  int rc = dsp_csr_alloc(m, g->num_cols, end - start, local);
  if (rc) return rc;
  for (int64_t i = 0; i <= m; ++i) local->indptr[i] = g->indptr[lb + i] - start;
  memcpy(local->indices, g->indices + start, sizeof(int64_t) * (size_t)(end - start));
  memcpy(local->values, g->values + start, sizeof(float) * (size_t)(end - start));
  return DSP_OK;
}
