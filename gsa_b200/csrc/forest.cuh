// SPDX-License-Identifier: Apache-2.0
// Host-side forest object: a batch of independent prefix BVHs (one per scene)
// built and queried together.  A single-scene tree is a forest of one.
#pragma once
#include <vector>
#include "common.cuh"

namespace gsa {

struct BuildScratch;

struct Forest {
  int B = 0;        // trees
  int N = 0;        // total support points
  int levels = 1;   // 4 for prefix trees
  int leaf = 16;    // maximum leaf size used by the builder
  int max_n = 0;
  long long q_total = 0;
  std::vector<TreeDesc> hdesc;
  TreeDesc* desc = nullptr;
  float4* pts = nullptr;
  float4* lpts = nullptr;  // level 1.. member arrays (prefix trees)
  Entry* nodes = nullptr;
  Entry* root = nullptr;
  int* qorder = nullptr;
  int* wrank = nullptr;
  int* cut = nullptr;
  int* ovf = nullptr;  // [0, B): capacity overflow flags; [B, 2B): kept counts
  void* block = nullptr;  // the one pool allocation holding the arrays above
  const float* x = nullptr;  // borrowed
  BuildScratch* scratch = nullptr;  // kept build temporaries (rebuild_forest)

  ForestView view() const {
    ForestView v;
    v.desc = desc;
    v.pts = pts;
    v.lpts = lpts;
    v.nodes = nodes;
    v.root = root;
    v.qorder = qorder;
    v.wrank = wrank;
    v.cut = cut;
    v.ovf = ovf;
    v.x = x;
    v.levels = levels;
    return v;
  }
};

// Builds a forest over `B` trees whose points are x[seg[b]*3 .. seg[b+1]*3)
// (seg on the host, B+1 entries, every tree non-empty).  Stream-ordered; no
// host synchronisation.  Returns cudaSuccess or an error.
cudaError_t build_forest(const float* x, const int* seg, int B, int prefix,
                         int leaf, cudaStream_t s, Forest** out);
cudaError_t free_forest(Forest* f, cudaStream_t s);
// Rebuilds `f` in place from points `x` with the same layout (scene sizes,
// levels, leaf size).  The first call allocates the build temporaries and
// keeps them with the forest; later calls allocate nothing, so a rebuild can
// be captured in a CUDA graph.  Stream-ordered; no host synchronisation.
cudaError_t rebuild_forest(Forest* f, const float* x, cudaStream_t s);

// Queries of one launch.  Single tree: qseg == qseg_host == qstart == null,
// `nq` queries at q[0..nq).  Forest: tree b answers qseg[b+1]-qseg[b] queries
// read from rows q[qstart[b]..) (qstart null: from row qseg[b]) and written to
// output rows qseg[b]..; qseg_host is the host copy of qseg.
struct QuerySet {
  const float* q = nullptr;
  const int* qstart = nullptr;
  const int* qseg = nullptr;
  const int* qseg_host = nullptr;
  int nq = 0;
  int m = 0;      // support prefix of every tree; 0 = that tree's level size
  int level = -1; // bounds level; -1 = all points
  bool morton = false;  // single tree: walk the queries in their own Morton
                        // order (they are not the support's points)
};

// Morton order of n query points q[0..n) (over their own finite bounds, as
// a tree's points are ordered before its build): enqueues the key sort and
// sets *perm to a device array of the n row indices in that order, which
// lives in *block (a pool allocation the caller frees, stream-ordered, once
// the queries that read it are enqueued).  build.cu.
cudaError_t sort_query_rows(const float* q, int n, const int** perm,
                            void** block, cudaStream_t s);

// Query launchers (query.cu).
cudaError_t launch_radius(const Forest& f, const QuerySet& qs, float radius,
                          int ns, int* out, int* fallback, cudaStream_t s);
cudaError_t launch_knn3(const Forest& f, const QuerySet& qs, float* d, int* ix,
                        int* fallback, cudaStream_t s);

}  // namespace gsa
