// threshold_probe.cu — TEST INFRASTRUCTURE ONLY (host code, no GPU needed).
//
// The reference evaluates its adaptive-selector threshold in a .cu translation unit
// compiled by nvcc (src/comm_man.h:396-400): float k, float u, and an unqualified
// pow(k, u). This probe evaluates the same expression form with the same types under nvcc,
// so the golden thresholds reflect nvcc's overload resolution and float arithmetic.
// Usage: threshold_probe a b c u dims...   -> prints one "dims threshold_hex" line per dims
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>

int main(int argc, char **argv) {
  if (argc < 6) return 2;
  float a = (float)atof(argv[1]), b = (float)atof(argv[2]), c = (float)atof(argv[3]), u = (float)atof(argv[4]);
  for (int i = 5; i < argc; ++i) {
    int dims = atoi(argv[i]);
    float k = std::min((float)c, (float)dims);
    float thr = 1 / (a * pow(k, u) + b / k);
    unsigned bits;
    memcpy(&bits, &thr, 4);
    printf("%d %08x\n", dims, bits);
  }
  return 0;
}
