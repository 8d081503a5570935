// SPDX-License-Identifier: Apache-2.0
// Per-library count of issued kernel launches, so callers (the benchmark) can
// report how many of this library's kernels ran in a timed region.
#include <atomic>
#include "common.cuh"

namespace gsa {
namespace {
std::atomic<unsigned long long> g_launches{0};
}
void count_launches(int n) { g_launches.fetch_add((unsigned long long)n); }
}  // namespace gsa

// See include/gsa_bvh.h and include/reference_queries.h.
GSA_API int launch_counter(unsigned long long* total) {
  if (!total) return -2;
  *total = gsa::g_launches.load();
  return 0;
}
