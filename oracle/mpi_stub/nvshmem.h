/* nvshmem.h — stand-in for the NVSHMEM declarations the reference's src/utils.h names.
 * TEST INFRASTRUCTURE ONLY (see mpi.h beside it): the golden runs never initialise NVSHMEM;
 * the functions abort if reached. */
#ifndef DSP_ORACLE_NVSHMEM_STUB_H
#define DSP_ORACLE_NVSHMEM_STUB_H
#include <cstdio>
#include <cstdlib>
#include "mpi.h"
#define NVSHMEMX_SUCCESS 0
#define NVSHMEMX_INIT_WITH_MPI_COMM 1
typedef struct {
  MPI_Comm *mpi_comm;
} nvshmemx_init_attr_t;
static inline int nvshmemx_init_attr(unsigned, nvshmemx_init_attr_t *) {
  fprintf(stderr, "nvshmem stub: not available\n");
  abort();
}
static inline void nvshmem_barrier_all() {
  fprintf(stderr, "nvshmem stub: not available\n");
  abort();
}
#endif
