// Test infrastructure only: a C entry point over the reference's own work
// partition (mlx-sparse src/common/cpu_parallel.cpp:202-253,
// weighted_cpu_ranges), compiled from the reference's source file where it
// lies into oracle/_ref/ by `make ref`. It checks the oracle's restatement
// of that partition (oracle.cpp weighted_ranges); nothing else links it.
#include <cstdint>
#include <vector>

#include "common/cpu_parallel.h"

extern "C" int ref_weighted_ranges(const int64_t *work, int64_t n, int parts, int64_t *out_pairs) {
  std::vector<int64_t> w(work, work + n);
  const auto ranges = mlx_sparse::weighted_cpu_ranges(w, parts);
  for (size_t i = 0; i < ranges.size(); ++i) {
    out_pairs[2 * i] = ranges[i].begin;
    out_pairs[2 * i + 1] = ranges[i].end;
  }
  return (int)ranges.size();
}
