// cli_dist_spmm_node.cpp — drop-in for the reference's dist_spmm_node / dist_spmm
// programs (src/dist_spmm_node.cu:20-444, src/dist_spmm.cu:19-491):
//
//   dist_spmm_node [-np P] <file_name> <dims> <task_dist> <comm_type> <n_rolls> <repeat>
//                  [nvlink_num_producers]
//
// The positional arguments and the report printed on stdout are the reference's. Two ways
// to run P ranks:
//   - one process per rank, as the reference runs (`mpirun -np P dist_spmm_node ...`, also
//     srun or torchrun): the rank, world size and node-local rank come from the launcher's
//     environment (Open MPI, MPICH/Hydra, Slurm, torchrun), each process drives the GPU of
//     its local rank (src/utils.h:176-237) and the ranks meet in a directory under /dev/shm
//     (DSP_STORE_DIR overrides it) for the host collectives; rank 0 prints the report;
//   - `-np P` (or DSP_NP): all ranks in this process, on GPUs rank % (visible GPUs).
// nvlink_num_producers sets how many fetch streams run concurrently. B is filled with 1.0
// as in the reference (src/dist_spmm_node.cu:192) unless DSP_B_SEED is set. DSP_C_OUT=<p>
// writes each rank's rows of C to <p>.<rank> (raw fp32, row-major) for checking.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <iomanip>
#include <iostream>
#include <string>
#include <vector>

#include "../../include/distspmm.h"

namespace {

int env_int(const char *name, int dflt) {
  const char *v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

// (rank, world, local rank) from the launcher's environment; world = 1 when none is set.
void launcher_rank(int *rank, int *world, int *local) {
  static const char *kVars[][3] = {
      {"OMPI_COMM_WORLD_RANK", "OMPI_COMM_WORLD_SIZE", "OMPI_COMM_WORLD_LOCAL_RANK"},  // Open MPI
      {"PMI_RANK", "PMI_SIZE", "MPI_LOCALRANKID"},                                      // MPICH / Hydra
      {"SLURM_PROCID", "SLURM_NTASKS", "SLURM_LOCALID"},                                // srun
      {"RANK", "WORLD_SIZE", "LOCAL_RANK"},                                             // torchrun
  };
  for (auto &v : kVars) {
    if (getenv(v[0]) && getenv(v[1])) {
      *rank = env_int(v[0], 0);
      *world = env_int(v[1], 1);
      *local = env_int(v[2], *rank);
      return;
    }
  }
  *rank = 0;
  *world = 1;
  *local = 0;
}

// The directory the job's processes meet in: DSP_STORE_DIR, else one named after the
// launcher process they share (their parent on this node) and its start time, so that
// every rank derives the same name and no two jobs share one.
std::string store_dir() {
  if (const char *d = getenv("DSP_STORE_DIR")) return d;
  const long ppid = (long)getppid();
  std::string start = "0";
  if (FILE *f = fopen(("/proc/" + std::to_string(ppid) + "/stat").c_str(), "r")) {
    char buf[4096];
    size_t n = fread(buf, 1, sizeof buf - 1, f);
    fclose(f);
    buf[n] = 0;
    // field 22 (starttime), counted after the closing parenthesis of the command name
    if (char *p = strrchr(buf, ')')) {
      int field = 2;
      for (char *t = strtok(p + 1, " "); t; t = strtok(nullptr, " "))
        if (++field == 22) {
          start = t;
          break;
        }
    }
  }
  return "/dev/shm/dsp_store_" + std::to_string(ppid) + "_" + start;
}

void print_report(const dsp_args &a, const std::string &file, const dsp_report &r) {
  std::cout << "task_distribution: " << a.task_dist << " and rolls:" << a.n_rolls << std::endl;
  for (int i = 0; i < r.T; ++i) std::cout << r.remap[i] << " ";
  std::cout << std::endl;
  std::cout << "Running dist_spmm programs on " << file << " with [" << a.dims << "] dims" << std::endl;
  std::cout << std::fixed << std::setprecision(3);
  std::cout << "Processing time: (ms) " << std::endl;
  std::cout << "Re-allocation time(all): " << r.stage_ms[3] << " Hira Time: " << r.hsdma_ms << std::endl;
  std::cout << "Max memory used: " << r.mem_gb << " GB" << std::endl;
  std::cout << "Average time used: " << r.avg_ms << " ms" << std::endl;
  std::cout << "Communication Traffic Intra : " << r.traffic_intra / (1024.0 * 1024.0 * 1024.0) << " GB" << std::endl;
  std::cout << "Communication Traffic Inter : " << r.traffic_inter / (1024.0 * 1024.0 * 1024.0) << " GB" << std::endl;
  std::cout << "Throughput: " << r.gflops << " GFLOPS" << std::endl;
}

}  // namespace

int main(int argc, char **argv) {
  int np_flag = 0;
  int np = getenv("DSP_NP") ? atoi(getenv("DSP_NP")) : 1;
  std::vector<char *> pos;
  for (int i = 1; i < argc; ++i) {
    if (strcmp(argv[i], "-np") == 0 && i + 1 < argc) {
      np = atoi(argv[++i]);
      np_flag = 1;
      continue;
    }
    pos.push_back(argv[i]);
  }
  if (pos.size() < 6) {
    std::cerr << "Usage: ./dist_spmm_node <file_name> <dims> <task_dist> <comm_type> <n_rolls> <repeat> "
              << std::endl;
    return EXIT_FAILURE;
  }
  dsp_args a;
  memset(&a, 0, sizeof a);
  std::string file = pos[0];
  try {
    a.dims = std::stoi(pos[1]);
    a.task_dist = std::stoi(pos[2]);
    a.comm_type = std::stoi(pos[3]);
    a.n_rolls = std::stoi(pos[4]);
    a.repeat = std::stoi(pos[5]);
    a.n_streams = pos.size() >= 7 ? std::stoi(pos[6]) : 4;
  } catch (const std::exception &e) {
    std::cerr << "bad argument: " << e.what() << std::endl;
    return EXIT_FAILURE;
  }
  if (file.size() >= 4 && file.substr(file.size() - 4) == ".mtx") {
    std::cout << "SparseMatrix::load_from_mtx not implemented" << std::endl;
    std::cerr << "Failed to load the matrix from the mtx file." << std::endl;
    return EXIT_FAILURE;
  }
  int ngpu = dsp_device_count();
  if (ngpu < 1) {
    std::cerr << "no CUDA device" << std::endl;
    return EXIT_FAILURE;
  }
  a.platform = DSP_PLATFORM_H100;
  if (const char *pf = getenv("DSP_PLATFORM")) {
    if (!strcmp(pf, "a800")) a.platform = DSP_PLATFORM_A800;
    if (!strcmp(pf, "b200")) a.platform = DSP_PLATFORM_B200;
  }
  a.b_ones = getenv("DSP_B_SEED") ? 0 : 1;
  a.b_seed = getenv("DSP_B_SEED") ? strtoull(getenv("DSP_B_SEED"), nullptr, 10) : 0;
  a.file = file.c_str();

  int rank = 0, world = 1, local = 0;
  launcher_rank(&rank, &world, &local);
  if (world > 1 && !np_flag && !getenv("DSP_NP")) {
    // one process per rank (mpirun -np P): this process is `rank`, on its local GPU
    dsp_store *st = nullptr;
    const double timeout_s = getenv("DSP_STORE_TIMEOUT_S") ? atof(getenv("DSP_STORE_TIMEOUT_S")) : 300.0;
    int rc = dsp_store_open(store_dir().c_str(), rank, world, timeout_s, &st);
    dsp_report r;
    std::vector<float> c_rows;
    const char *c_out = getenv("DSP_C_OUT");
    if (rc == DSP_OK && c_out) {
      int64_t M = 0, lb = 0, ub = 0;
      if ((rc = dsp_csr_read_indptr(a.file, &M, nullptr)) == DSP_OK) {
        std::vector<int64_t> ip;
        const char *part = getenv("DSP_PARTITION");
        if (part && !strcmp(part, "balanced")) {
          ip.resize((size_t)M + 1);
          rc = dsp_csr_read_indptr(a.file, &M, ip.data());
          if (rc == DSP_OK) rc = dsp_partition_bounds_balanced(ip.data(), M, world, rank, &lb, &ub);
        } else {
          rc = dsp_partition_bounds(M, world, rank, &lb, &ub);
        }
        c_rows.resize((size_t)std::max<int64_t>(ub - lb, 1) * (size_t)a.dims);
        a.c_out = c_rows.data();
      }
    }
    if (rc == DSP_OK) rc = dsp_run_rank(&a, rank, world, local % ngpu, st, &r);
    if (rc != DSP_OK) {
      std::cerr << "dist_spmm_node rank " << rank << " failed (" << rc << "): " << dsp_last_error() << std::endl;
      dsp_store_close(st, 0);
      return EXIT_FAILURE;
    }
    if (c_out) {
      const std::string path = std::string(c_out) + "." + std::to_string(rank);
      FILE *f = fopen(path.c_str(), "wb");
      const size_t n = (size_t)(r.row_ub - r.row_lb) * (size_t)a.dims;
      if (!f || fwrite(c_rows.data(), 4, n, f) != n) {
        std::cerr << "cannot write " << path << std::endl;
        if (f) fclose(f);
        dsp_store_close(st, 0);
        return EXIT_FAILURE;
      }
      fclose(f);
    }
    if (rank == 0) print_report(a, file, r);
    dsp_store_close(st, 1);
    return EXIT_SUCCESS;
  }

  if (np < 1) np = 1;
  std::vector<int> devices((size_t)np);
  for (int p = 0; p < np; ++p) devices[(size_t)p] = p % ngpu;
  a.world = np;
  a.devices = devices.data();
  dsp_report r;
  int rc = dsp_run(&a, &r);
  if (rc != DSP_OK) {
    std::cerr << "dist_spmm_node failed (" << rc << "): " << dsp_last_error() << std::endl;
    return EXIT_FAILURE;
  }
  print_report(a, file, r);
  return EXIT_SUCCESS;
}
