// store.cpp — host collectives for ranks launched as separate processes on one node.
//
// The reference runs one MPI process per GPU and does its host collectives with MPI
// (Gather / Bcast of the HSDMA demand, src/utils.h:358-437; Allgather(v) of the needed
// sets, src/utils.h:439-547; Allreduce of the statistics, src/dist_spmm_node.cu:401-409).
// No MPI library exists in this build's environment, and one node needs none: the ranks
// meet in a directory (tmpfs on Linux) that every process of the job can reach. A rank
// publishes a value by writing <dir>/<key>.<rank> under a temporary name and renaming it
// (readers see the whole file or none); it collects the others' values by polling for
// their files with a bounded wait, so a rank that died or never started makes the others
// fail with DSP_ERR_TIMEOUT instead of hanging. Keys are used once per run.
#include <dirent.h>
#include <errno.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <string>

#include "internal.h"

using namespace dsp;

struct dsp_store {
  std::string dir;
  int rank = 0, world = 1;
  double timeout_s = 300.0;

  std::string path(const char *key, int r) const { return dir + "/" + key + "." + std::to_string(r); }

  int put(const char *key, const void *data, size_t n) {
    const std::string p = path(key, rank), tmp = p + ".part";
    FILE *f = fopen(tmp.c_str(), "wb");
    if (!f) return fail(DSP_ERR_IO, "store: cannot create %s: %s", tmp.c_str(), strerror(errno));
    const size_t w = n ? fwrite(data, 1, n, f) : 0;
    if (fclose(f) != 0 || w != n) return fail(DSP_ERR_IO, "store: short write of %s", tmp.c_str());
    if (rename(tmp.c_str(), p.c_str()) != 0)
      return fail(DSP_ERR_IO, "store: rename to %s: %s", p.c_str(), strerror(errno));
    return DSP_OK;
  }

  // Wait (bounded) for rank r's value under key and read it.
  int get(const char *key, int r, std::string *out) {
    using clock = std::chrono::steady_clock;
    const auto t0 = clock::now();
    const std::string p = path(key, r);
    useconds_t pause = 50;
    for (;;) {
      FILE *f = fopen(p.c_str(), "rb");
      if (f) {
        out->clear();
        char buf[1 << 16];
        size_t k;
        while ((k = fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, k);
        fclose(f);
        return DSP_OK;
      }
      if (std::chrono::duration<double>(clock::now() - t0).count() > timeout_s)
        return fail(DSP_ERR_TIMEOUT, "store: rank %d waited %.0f s for '%s' of rank %d (rank gone or not started)",
                    rank, timeout_s, key, r);
      usleep(pause);
      pause = pause < 20000 ? pause * 2 : 20000;
    }
  }
};

extern "C" int dsp_store_open(const char *dir, int rank, int world, double timeout_s, dsp_store **out) {
  DSP_TRY_ARG(dir && *dir && out, "dsp_store_open: null argument");
  DSP_TRY_ARG(world >= 1 && rank >= 0 && rank < world, "dsp_store_open: rank %d of %d", rank, world);
  *out = nullptr;
  if (mkdir(dir, 0700) != 0 && errno != EEXIST)
    return fail(DSP_ERR_IO, "dsp_store_open: mkdir %s: %s", dir, strerror(errno));
  dsp_store *s = new dsp_store();
  s->dir = dir;
  s->rank = rank;
  s->world = world;
  if (timeout_s > 0) s->timeout_s = timeout_s;
  *out = s;
  return DSP_OK;
}

extern "C" int dsp_store_allgather(dsp_store *s, const char *key, const void *data, int64_t bytes, void *out,
                                   int64_t out_cap, int64_t *sizes) {
  DSP_TRY_ARG(s && key && *key && strchr(key, '/') == nullptr && bytes >= 0 && (data || bytes == 0),
              "dsp_store_allgather: bad argument");
  int rc = s->put(key, data, (size_t)bytes);
  if (rc) return rc;
  int64_t off = 0;
  std::string v;
  for (int r = 0; r < s->world; ++r) {
    if ((rc = s->get(key, r, &v))) return rc;
    if (sizes) sizes[r] = (int64_t)v.size();
    if (out) {
      if (off + (int64_t)v.size() > out_cap)
        return fail(DSP_ERR_INVALID, "dsp_store_allgather: '%s' needs more than %lld bytes", key,
                    (long long)out_cap);
      memcpy((char *)out + off, v.data(), v.size());
    }
    off += (int64_t)v.size();
  }
  return DSP_OK;
}

extern "C" int dsp_store_barrier(dsp_store *s, const char *key) {
  return dsp_store_allgather(s, key, nullptr, 0, nullptr, 0, nullptr);
}

extern "C" void dsp_store_close(dsp_store *s, int remove_dir) {
  if (!s) return;
  if (remove_dir) {
    // Every rank has passed the caller's last collective once all "bye" files exist, so
    // rank 0 then removes the directory; the others leave right after saying bye.
    const bool ok = s->put("bye", nullptr, 0) == DSP_OK;
    if (ok && s->rank == 0) {
      std::string v;
      bool all = true;
      for (int r = 0; r < s->world && all; ++r) all = s->get("bye", r, &v) == DSP_OK;
      if (all) {
        if (DIR *d = opendir(s->dir.c_str())) {
          while (dirent *e = readdir(d))
            if (strcmp(e->d_name, ".") && strcmp(e->d_name, "..")) unlink((s->dir + "/" + e->d_name).c_str());
          closedir(d);
        }
        rmdir(s->dir.c_str());
      }
    }
  }
  delete s;
}
