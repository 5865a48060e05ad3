// host_gen.cpp — seeded synthetic inputs: R-MAT, 27-point stencil, uniform random
// matrices, and the dense B values. All generators are counter-based (every value is a
// hash of (seed, position)), so the output does not depend on the host thread count.
#include <string.h>

#include "internal.h"

using namespace dsp;

namespace {

const uint64_t kValueSalt = 0x5EEDF00DBAADC0DEull;

// Row-wise sort + dedup of a CSR whose rows hold unsorted, possibly repeated column ids;
// fills `out` with the compacted matrix and values U(0,1) = hash(seed, row, col).
int compact_rows(int64_t n, const std::vector<int64_t> &ptr, std::vector<int32_t> &cols, uint64_t seed,
                 dsp_csr *out) {
  std::vector<int64_t> uniq((size_t)n + 1, 0);
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      int32_t *s = cols.data() + ptr[r], *t = cols.data() + ptr[r + 1];
      std::sort(s, t);
      uniq[r + 1] = std::unique(s, t) - s;
    }
  }, 1024);
  for (int64_t r = 0; r < n; ++r) uniq[r + 1] += uniq[r];
  int rc = dsp_csr_alloc(n, n, uniq[n], out);
  if (rc) return rc;
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r <= e - 1; ++r) {
      out->indptr[r + 1] = uniq[r + 1];
      const int64_t cnt = uniq[r + 1] - uniq[r];
      for (int64_t k = 0; k < cnt; ++k) {
        int64_t c = cols[ptr[r] + k];
        out->indices[uniq[r] + k] = c;
        out->values[uniq[r] + k] = u01_24(hash3(seed ^ kValueSalt, (uint64_t)r, (uint64_t)c));
      }
    }
  }, 1024);
  out->indptr[0] = 0;
  return DSP_OK;
}

// One R-MAT edge: per level (most significant bit first) pick a quadrant with
// probabilities a, b, c, d from 32 random bits.
inline void rmat_edge(uint64_t seed, uint64_t e, int scale, double a, double ab, double abc, int64_t *pi,
                      int64_t *pj) {
  int64_t i = 0, j = 0;
  uint64_t bits = 0;
  for (int l = 0; l < scale; ++l) {
    if ((l & 1) == 0) bits = hash3(seed, e, (uint64_t)l);
    double r = (double)(uint32_t)(bits >> ((l & 1) * 32)) * (1.0 / 4294967296.0);
    int bi = 0, bj = 0;
    if (r < a) {
    } else if (r < ab) {
      bj = 1;
    } else if (r < abc) {
      bi = 1;
    } else {
      bi = 1;
      bj = 1;
    }
    i = (i << 1) | bi;
    j = (j << 1) | bj;
  }
  *pi = i;
  *pj = j;
}

}  // namespace

extern "C" int dsp_gen_rmat(int scale, int edge_factor, double a, double b, double c, uint64_t seed,
                            dsp_csr *out) {
  DSP_TRY_ARG(out, "dsp_gen_rmat: out is NULL");
  DSP_TRY_ARG(scale >= 1 && scale <= 30 && edge_factor >= 1, "dsp_gen_rmat: scale %d / edge factor %d", scale,
              edge_factor);
  DSP_TRY_ARG(a >= 0 && b >= 0 && c >= 0 && a + b + c <= 1.0, "dsp_gen_rmat: bad probabilities");
  const int64_t n = (int64_t)1 << scale;
  const int64_t E = (int64_t)edge_factor * n;
  const double ab = a + b, abc = a + b + c;
  std::vector<int64_t> deg((size_t)n + 1, 0);
  // pass 1: degrees of the symmetrised edge list (self-loops dropped)
  parallel_for(E, [&](int64_t lo, int64_t hi) {
    for (int64_t e = lo; e < hi; ++e) {
      int64_t i, j;
      rmat_edge(seed, (uint64_t)e, scale, a, ab, abc, &i, &j);
      if (i == j) continue;
      __atomic_fetch_add(&deg[i + 1], 1, __ATOMIC_RELAXED);
      __atomic_fetch_add(&deg[j + 1], 1, __ATOMIC_RELAXED);
    }
  }, 1 << 16);
  for (int64_t r = 0; r < n; ++r) deg[r + 1] += deg[r];
  std::vector<int32_t> cols((size_t)std::max<int64_t>(deg[n], 1));
  std::vector<int64_t> cur(deg.begin(), deg.end() - 1);
  // pass 2: scatter both directions (order inside a row is fixed by the sort below)
  parallel_for(E, [&](int64_t lo, int64_t hi) {
    for (int64_t e = lo; e < hi; ++e) {
      int64_t i, j;
      rmat_edge(seed, (uint64_t)e, scale, a, ab, abc, &i, &j);
      if (i == j) continue;
      cols[__atomic_fetch_add(&cur[i], 1, __ATOMIC_RELAXED)] = (int32_t)j;
      cols[__atomic_fetch_add(&cur[j], 1, __ATOMIC_RELAXED)] = (int32_t)i;
    }
  }, 1 << 16);
  return compact_rows(n, deg, cols, seed, out);
}

extern "C" int dsp_gen_stencil27(int64_t n, uint64_t seed, dsp_csr *out) {
  DSP_TRY_ARG(out && n >= 1 && n <= 1200, "dsp_gen_stencil27: grid %lld", (long long)n);
  const int64_t M = n * n * n;
  auto span = [n](int64_t v) { return (int64_t)(v > 0) + 1 + (int64_t)(v < n - 1); };
  std::vector<int64_t> ptr((size_t)M + 1, 0);
  parallel_for(M, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      int64_t x = r % n, y = (r / n) % n, z = r / (n * n);
      ptr[r + 1] = span(x) * span(y) * span(z);
    }
  });
  for (int64_t r = 0; r < M; ++r) ptr[r + 1] += ptr[r];
  int rc = dsp_csr_alloc(M, M, ptr[M], out);
  if (rc) return rc;
  memcpy(out->indptr, ptr.data(), sizeof(int64_t) * (size_t)(M + 1));
  parallel_for(M, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      int64_t x = r % n, y = (r / n) % n, z = r / (n * n);
      int64_t p = ptr[r];
      for (int dz = -1; dz <= 1; ++dz) {
        if (z + dz < 0 || z + dz >= n) continue;
        for (int dy = -1; dy <= 1; ++dy) {
          if (y + dy < 0 || y + dy >= n) continue;
          for (int dx = -1; dx <= 1; ++dx) {
            if (x + dx < 0 || x + dx >= n) continue;
            int64_t c = r + dz * n * n + dy * n + dx;
            out->indices[p] = c;
            out->values[p] = (c == r) ? 26.0f : -u01_24(hash3(seed ^ kValueSalt, (uint64_t)r, (uint64_t)c));
            ++p;
          }
        }
      }
    }
  });
  return DSP_OK;
}

extern "C" int dsp_gen_uniform(int64_t rows, int64_t k, uint64_t seed, dsp_csr *out) {
  DSP_TRY_ARG(out && rows >= 1 && k >= 0 && k <= rows && k <= 4096, "dsp_gen_uniform: %lld rows, %lld per row",
              (long long)rows, (long long)k);
  int rc = dsp_csr_alloc(rows, rows, rows * k, out);
  if (rc) return rc;
  for (int64_t r = 0; r <= rows; ++r) out->indptr[r] = r * k;
  parallel_for(rows, [&](int64_t b, int64_t e) {
    std::vector<int64_t> pick((size_t)k);
    for (int64_t r = b; r < e; ++r) {
      int64_t got = 0;
      uint64_t attempt = 0;
      while (got < k) {
        int64_t c = (int64_t)(hash3(seed, (uint64_t)r, attempt++) % (uint64_t)rows);
        bool dup = false;
        for (int64_t q = 0; q < got; ++q)
          if (pick[q] == c) {
            dup = true;
            break;
          }
        if (!dup) pick[got++] = c;
      }
      std::sort(pick.begin(), pick.end());
      for (int64_t q = 0; q < k; ++q) {
        out->indices[r * k + q] = pick[q];
        out->values[r * k + q] = u01_24(hash3(seed ^ kValueSalt, (uint64_t)r, (uint64_t)pick[q]));
      }
    }
  }, 1024);
  return DSP_OK;
}

extern "C" int dsp_fill_dense_host(float *B, int64_t row0, int64_t rows, int64_t ld, int64_t ncols, uint64_t seed) {
  DSP_TRY_ARG(B && rows >= 0 && ncols >= 0 && ld >= ncols, "dsp_fill_dense_host: bad argument");
  parallel_for(rows, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r)
      for (int64_t c = 0; c < ncols; ++c) B[r * ld + c] = dense_value(seed, row0 + r, c);
  }, 256);
  return DSP_OK;
}

extern "C" int dsp_fill_dense_rows_host(float *B, const int64_t *rows, int64_t n, int64_t ld, int64_t ncols,
                                        uint64_t seed) {
  DSP_TRY_ARG(B && (rows || n == 0) && n >= 0 && ncols >= 0 && ld >= ncols, "dsp_fill_dense_rows_host: bad argument");
  parallel_for(n, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i)
      for (int64_t c = 0; c < ncols; ++c) B[i * ld + c] = dense_value(seed, rows[i], c);
  }, 256);
  return DSP_OK;
}
