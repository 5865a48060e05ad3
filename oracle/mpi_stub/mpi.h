/* mpi.h — a single-process stand-in for the MPI calls the reference's host code makes.
 *
 * TEST INFRASTRUCTURE ONLY: it exists so that the reference's own MPI-bound functions
 * (double_level_comm_node_processing and ComputeAllocation_HSDMA_MPI of src/utils.h) can be
 * compiled here, where no MPI library exists, and run to produce golden vectors. The ranks
 * of one job are threads of one process (one node): every collective publishes each rank's
 * buffer pointer, meets at a barrier, copies what the call's semantics say, and meets again.
 * Only the calls and constants the reference's src/utils.h names are provided; the ones the
 * golden runs never reach abort. */
#ifndef DSP_ORACLE_MPI_STUB_H
#define DSP_ORACLE_MPI_STUB_H

#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

typedef int MPI_Comm;
typedef int MPI_Datatype;
typedef int MPI_Info;
typedef int MPI_Op;

#define MPI_SUCCESS 0
#define MPI_COMM_WORLD 0
#define MPI_COMM_NULL (-1)
#define MPI_INFO_NULL 0
#define MPI_COMM_TYPE_SHARED 1
#define MPI_UNDEFINED (-32766)
#define MPI_MAX_ERROR_STRING 256
#define MPI_INT 4
#define MPI_FLOAT 104
#define MPI_LONG 8
#define MPI_DOUBLE 108
#define MPI_CHAR 1

namespace dsp_mpi_stub {

struct World {
  int size = 1;
  std::mutex mu;
  std::condition_variable cv;
  int count = 0;
  long gen = 0;
  std::vector<const void *> ptr;
  std::vector<const int *> counts, displs;
  void barrier() {
    std::unique_lock<std::mutex> lk(mu);
    const long g = gen;
    if (++count == size) {
      count = 0;
      ++gen;
      cv.notify_all();
    } else {
      cv.wait(lk, [&] { return gen != g; });
    }
  }
};

inline World &world() {
  static World w;
  return w;
}
inline int &rank() {
  static thread_local int r = 0;
  return r;
}
inline size_t type_size(MPI_Datatype t) { return t >= 100 ? (size_t)(t - 100) : (size_t)t; }

/* Run fn(rank) on `size` threads, one per rank (the job's processes on one node). */
template <class F>
void run_ranks(int size, F fn);

}  // namespace dsp_mpi_stub

static inline int MPI_Comm_rank(MPI_Comm, int *r) {
  *r = dsp_mpi_stub::rank();
  return MPI_SUCCESS;
}
static inline int MPI_Comm_size(MPI_Comm, int *s) {
  *s = dsp_mpi_stub::world().size;
  return MPI_SUCCESS;
}
/* one node: the shared-memory communicator is the world */
static inline int MPI_Comm_split_type(MPI_Comm comm, int, int, MPI_Info, MPI_Comm *out) {
  *out = comm;
  return MPI_SUCCESS;
}
static inline int MPI_Comm_split(MPI_Comm, int, int, MPI_Comm *) {
  fprintf(stderr, "mpi stub: MPI_Comm_split is not provided\n");
  abort();
}
static inline int MPI_Comm_free(MPI_Comm *) { return MPI_SUCCESS; }
static inline int MPI_Initialized(int *f) {
  *f = 1;
  return MPI_SUCCESS;
}
static inline int MPI_Error_string(int code, char *s, int *len) {
  *len = snprintf(s, MPI_MAX_ERROR_STRING, "mpi stub error %d", code);
  return MPI_SUCCESS;
}
static inline double MPI_Wtime() {
  return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}
static inline int MPI_Barrier(MPI_Comm) {
  dsp_mpi_stub::world().barrier();
  return MPI_SUCCESS;
}
static inline int MPI_Allgather(const void *sbuf, int scount, MPI_Datatype stype, void *rbuf, int rcount,
                                MPI_Datatype rtype, MPI_Comm) {
  auto &w = dsp_mpi_stub::world();
  const int me = dsp_mpi_stub::rank();
  w.ptr[(size_t)me] = sbuf;
  w.barrier();
  const size_t bytes = (size_t)scount * dsp_mpi_stub::type_size(stype);
  for (int r = 0; r < w.size; ++r)
    memcpy((char *)rbuf + (size_t)r * rcount * dsp_mpi_stub::type_size(rtype), w.ptr[(size_t)r], bytes);
  w.barrier();
  return MPI_SUCCESS;
}
static inline int MPI_Allgatherv(const void *sbuf, int scount, MPI_Datatype stype, void *rbuf, const int *rcounts,
                                 const int *displs, MPI_Datatype rtype, MPI_Comm) {
  auto &w = dsp_mpi_stub::world();
  const int me = dsp_mpi_stub::rank();
  (void)scount;
  (void)stype;
  w.ptr[(size_t)me] = sbuf;
  w.barrier();
  const size_t ts = dsp_mpi_stub::type_size(rtype);
  for (int r = 0; r < w.size; ++r)
    if (rcounts[r] > 0) memcpy((char *)rbuf + (size_t)displs[r] * ts, w.ptr[(size_t)r], (size_t)rcounts[r] * ts);
  w.barrier();
  return MPI_SUCCESS;
}
static inline int MPI_Gather(const void *sbuf, int scount, MPI_Datatype stype, void *rbuf, int rcount,
                             MPI_Datatype rtype, int root, MPI_Comm) {
  auto &w = dsp_mpi_stub::world();
  const int me = dsp_mpi_stub::rank();
  w.ptr[(size_t)me] = sbuf;
  w.barrier();
  if (me == root)
    for (int r = 0; r < w.size; ++r)
      memcpy((char *)rbuf + (size_t)r * rcount * dsp_mpi_stub::type_size(rtype), w.ptr[(size_t)r],
             (size_t)scount * dsp_mpi_stub::type_size(stype));
  w.barrier();
  return MPI_SUCCESS;
}
static inline int MPI_Bcast(void *buf, int count, MPI_Datatype type, int root, MPI_Comm) {
  auto &w = dsp_mpi_stub::world();
  const int me = dsp_mpi_stub::rank();
  if (me == root) w.ptr[(size_t)root] = buf;
  w.barrier();
  if (me != root) memcpy(buf, w.ptr[(size_t)root], (size_t)count * dsp_mpi_stub::type_size(type));
  w.barrier();
  return MPI_SUCCESS;
}

#include <thread>

template <class F>
void dsp_mpi_stub::run_ranks(int size, F fn) {
  auto &w = world();
  w.size = size;
  w.count = 0;
  w.ptr.assign((size_t)size, nullptr);
  std::vector<std::thread> th;
  for (int r = 0; r < size; ++r)
    th.emplace_back([r, &fn] {
      rank() = r;
      fn(r);
    });
  for (auto &t : th) t.join();
}

#endif
