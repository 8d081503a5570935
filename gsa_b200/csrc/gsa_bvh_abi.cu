// SPDX-License-Identifier: Apache-2.0
// C ABI of libgsa_bvh: the exports GSA's gsa/runtime.py binds
// (csrc/gsa_bvh.cu:217-383) plus forest (multi-scene) extensions.
// Declarations and the reference interface each one replaces:
// include/gsa_bvh.h.
#include <algorithm>
#include "forest.cuh"
#include "pool.cuh"

using namespace gsa;

namespace {

int as_code(cudaError_t e) { return (int)e; }

// Bounds level l is exact for prefixes up to its size; a larger support
// prefix would make the level's boxes non-conservative.
bool level_ok(const Forest* f, int m, int level) {
  if (level < -1 || level >= kMaxLevels) return false;
  if (level >= f->levels) return false;
  if (f->B != 1) return false;
  return m <= level_size(f->hdesc[0].n, level);
}

}  // namespace

GSA_API int build_bvh(const float* x, int n, int prefix, int leaf, void** out,
                      void* stream) {
  if (!out || !x || n < 1 || n > kMaxPoints || leaf < 1) return -1;
  int seg[2] = {0, n};
  Forest* f = nullptr;
  cudaError_t e = build_forest(x, seg, 1, prefix, leaf, (cudaStream_t)stream, &f);
  if (e == cudaErrorInvalidValue) return -1;
  if (e) return as_code(e);
  *out = f;
  return 0;
}

GSA_API int query_bvh(void* handle, const float* q, int nq, int m, int level,
                      float* d, int* ix, int* fallback, void* stream) {
  Forest* f = (Forest*)handle;
  if (!f || nq < 0 || m < 3 || m > f->hdesc[0].n || !level_ok(f, m, level))
    return -2;
  if (!nq) return 0;
  if (!q || !d || !ix || !fallback) return -2;
  QuerySet qs;
  qs.q = q;
  qs.nq = nq;
  qs.m = m;
  qs.level = level;
  return as_code(launch_knn3(*f, qs, d, ix, fallback, (cudaStream_t)stream));
}

GSA_API int query_ball_bvh(void* handle, const float* q, int nq, int m,
                           int level, float radius, int ns, int* out,
                           int* fallback, void* stream) {
  Forest* f = (Forest*)handle;
  if (!f || nq < 0 || m < 1 || m > f->hdesc[0].n || ns < 1 || ns > 32 ||
      !level_ok(f, m, level))
    return -2;
  if (!nq) return 0;
  if (!q || !out || !fallback) return -2;
  QuerySet qs;
  qs.q = q;
  qs.nq = nq;
  qs.m = m;
  qs.level = level;
  return as_code(
      launch_radius(*f, qs, radius, ns, out, fallback, (cudaStream_t)stream));
}

// As query_bvh / query_ball_bvh, walking the queries in their own Morton
// order (see include/gsa_bvh.h).
GSA_API int query_bvh_unordered(void* handle, const float* q, int nq, int m,
                                int level, float* d, int* ix, int* fallback,
                                void* stream) {
  Forest* f = (Forest*)handle;
  if (!f || nq < 0 || m < 3 || m > f->hdesc[0].n || !level_ok(f, m, level))
    return -2;
  if (!nq) return 0;
  if (!q || !d || !ix || !fallback) return -2;
  QuerySet qs;
  qs.q = q;
  qs.nq = nq;
  qs.m = m;
  qs.level = level;
  qs.morton = true;
  return as_code(launch_knn3(*f, qs, d, ix, fallback, (cudaStream_t)stream));
}

GSA_API int query_ball_bvh_unordered(void* handle, const float* q, int nq,
                                     int m, int level, float radius, int ns,
                                     int* out, int* fallback, void* stream) {
  Forest* f = (Forest*)handle;
  if (!f || nq < 0 || m < 1 || m > f->hdesc[0].n || ns < 1 || ns > 32 ||
      !level_ok(f, m, level))
    return -2;
  if (!nq) return 0;
  if (!q || !out || !fallback) return -2;
  QuerySet qs;
  qs.q = q;
  qs.nq = nq;
  qs.m = m;
  qs.level = level;
  qs.morton = true;
  return as_code(
      launch_radius(*f, qs, radius, ns, out, fallback, (cudaStream_t)stream));
}

GSA_API int free_bvh(void* handle, int async_free, void* stream) {
  Forest* f = (Forest*)handle;
  if (!f) return -3;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = free_forest(f, s);
  if (!e && !async_free) e = cudaStreamSynchronize(s);
  return as_code(e);
}

GSA_API int set_pool_mode(int enabled) {
  pool_set_enabled(enabled);
  return 0;
}

GSA_API int pool_memory(uint64_t* used, uint64_t* reserved) {
  if (!used || !reserved) return -2;
  return as_code(pool_peaks(used, reserved));
}

GSA_API int pool_reset_peak(void) { return as_code(pool_reset_peaks()); }

// ---------------------------------------------------------------------------
// Forest extensions (no counterpart in the reference): B independent scenes
// built and queried with one launch per build step / query.

GSA_API int build_bvh_batch(const float* x, const int* seg, int b, int prefix,
                            int leaf, void** out, void* stream) {
  if (!out || !x || !seg || b < 1 || leaf < 1) return -1;
  Forest* f = nullptr;
  cudaError_t e = build_forest(x, seg, b, prefix, leaf, (cudaStream_t)stream, &f);
  if (e == cudaErrorInvalidValue) return -1;
  if (e) return as_code(e);
  *out = f;
  return 0;
}

GSA_API int rebuild_bvh_batch(void* handle, const float* x, void* stream) {
  Forest* f = (Forest*)handle;
  if (!f || !x) return -1;
  return as_code(rebuild_forest(f, x, (cudaStream_t)stream));
}

namespace {
// Every tree with queries must have a support prefix of at least min_m
// points that its level's bounds cover.
int check_batch(const Forest* f, const int* qseg, const int* qseg_host, int m,
                int level, int min_m) {
  if (!f || !qseg || !qseg_host || m < 0 || level < -1 || level >= f->levels)
    return -2;
  if (qseg_host[0] != 0) return -2;
  for (int b = 0; b < f->B; ++b) {
    if (qseg_host[b + 1] < qseg_host[b]) return -2;
    if (qseg_host[b + 1] == qseg_host[b]) continue;
    int size = level_size(f->hdesc[b].n, level);
    int mb = m ? m : size;
    if (mb < min_m || mb > size) return -2;
  }
  return 0;
}

QuerySet batch_set(const float* q, const int* qstart, const int* qseg,
                   const int* qseg_host, int m, int level) {
  QuerySet qs;
  qs.q = q;
  qs.qstart = qstart;
  qs.qseg = qseg;
  qs.qseg_host = qseg_host;
  qs.m = m;
  qs.level = level;
  return qs;
}
}  // namespace

GSA_API int query_ball_bvh_batch(void* handle, const float* q,
                                 const int* qstart, const int* qseg,
                                 const int* qseg_host, int m, int level,
                                 float radius, int ns, int* out, int* fallback,
                                 void* stream) {
  Forest* f = (Forest*)handle;
  if (ns < 1 || ns > 32) return -2;
  int c = check_batch(f, qseg, qseg_host, m, level, 1);
  if (c) return c;
  if (qseg_host[f->B] == 0) return 0;
  if (!q || !out || !fallback) return -2;
  return as_code(launch_radius(*f, batch_set(q, qstart, qseg, qseg_host, m, level),
                               radius, ns, out, fallback, (cudaStream_t)stream));
}

GSA_API int query_bvh_batch(void* handle, const float* q, const int* qstart,
                            const int* qseg, const int* qseg_host, int m,
                            int level, float* d, int* ix, int* fallback,
                            void* stream) {
  Forest* f = (Forest*)handle;
  int c = check_batch(f, qseg, qseg_host, m, level, 3);
  if (c) return c;
  if (qseg_host[f->B] == 0) return 0;
  if (!q || !d || !ix || !fallback) return -2;
  return as_code(launch_knn3(*f, batch_set(q, qstart, qseg, qseg_host, m, level),
                             d, ix, fallback, (cudaStream_t)stream));
}

GSA_API int bvh_info(void* handle, int* trees, int* points, int* levels,
                     int* leaf) {
  Forest* f = (Forest*)handle;
  if (!f) return -2;
  if (trees) *trees = f->B;
  if (points) *points = f->N;
  if (levels) *levels = f->levels;
  if (leaf) *leaf = f->leaf;
  return 0;
}
