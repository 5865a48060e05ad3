// cli_dist_spmm_node.cpp — drop-in for the reference's dist_spmm_node / dist_spmm
// programs (src/dist_spmm_node.cu:20-444, src/dist_spmm.cu:19-491):
//
//   dist_spmm_node [-np P] <file_name> <dims> <task_dist> <comm_type> <n_rolls> <repeat>
//                  [nvlink_num_producers]
//
// The positional arguments and the report printed on stdout are the reference's. The
// reference takes P from `mpirun -np P`; here `-np P` (or DSP_NP) sets it and the ranks
// run in this process on GPUs rank % (visible GPUs). nvlink_num_producers sets how many
// fetch streams run concurrently. B is filled with 1.0 as in the reference
// (src/dist_spmm_node.cu:192) unless DSP_B_SEED is set.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <iomanip>
#include <iostream>
#include <string>
#include <vector>

#include "../../include/distspmm.h"

int main(int argc, char **argv) {
  int np = getenv("DSP_NP") ? atoi(getenv("DSP_NP")) : 1;
  std::vector<char *> pos;
  for (int i = 1; i < argc; ++i) {
    if (strcmp(argv[i], "-np") == 0 && i + 1 < argc) {
      np = atoi(argv[++i]);
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
  if (np < 1) np = 1;
  std::vector<int> devices((size_t)np);
  for (int p = 0; p < np; ++p) devices[(size_t)p] = p % ngpu;
  a.file = file.c_str();
  a.world = np;
  a.devices = devices.data();
  a.platform = DSP_PLATFORM_H100;
  if (const char *pf = getenv("DSP_PLATFORM")) {
    if (!strcmp(pf, "a800")) a.platform = DSP_PLATFORM_A800;
    if (!strcmp(pf, "b200")) a.platform = DSP_PLATFORM_B200;
  }
  a.b_ones = getenv("DSP_B_SEED") ? 0 : 1;
  a.b_seed = getenv("DSP_B_SEED") ? strtoull(getenv("DSP_B_SEED"), nullptr, 10) : 0;
  dsp_report r;
  int rc = dsp_run(&a, &r);
  if (rc != DSP_OK) {
    std::cerr << "dist_spmm_node failed (" << rc << "): " << dsp_last_error() << std::endl;
    return EXIT_FAILURE;
  }
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
  return EXIT_SUCCESS;
}
