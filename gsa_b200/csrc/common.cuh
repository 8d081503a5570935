// SPDX-License-Identifier: Apache-2.0
// Shared device-side definitions of the B200 query engine: the forest layout
// in HBM, the exact FP32 distance and the round-down box lower bound.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <limits.h>

#define GSA_API extern "C" __attribute__((visibility("default")))

namespace gsa {

// Kernel launches issued by this library (read with launch_counter()).
void count_launches(int n = 1);

constexpr int kMaxLevels = 4;   // prefixes n, n/4, n/16, n/64
constexpr int kCutMax = 32;    // cut entries per tree and level
constexpr int kCutStride = kCutMax + 1;  // count, then the entries
constexpr int kMaxLeaf = 32;    // leaf point count fits 5 bits
constexpr int kMaxPoints = 1 << 26;  // leaf start fits 26 bits
constexpr unsigned kFull = 0xffffffffu;

// One child entry of a binary node, per prefix level: 32 bytes, loaded as two
// float4.  `minid` is the smallest original support ID in the subtree (all
// levels); `ref` >= 0 names an internal node, ref < 0 encodes a leaf
// ~((start << 5) | (count - 1)) whose `count` points are this level's members.
// Level 0 leaves index `pts` (ascending ID inside a leaf).  On a level l >= 1
// every subtree with at most `leaf` members of that level is a leaf ("level
// leaf") indexing that level's member array (level_pts), where the members of
// any subtree are contiguous; inside a level leaf IDs ascend only within each
// level-0 leaf it spans.  An empty entry (no finite member) has lo > hi and is
// never entered.
struct Entry {
  float lox, loy, loz;
  int minid;
  float hix, hiy, hiz;
  int ref;
};
static_assert(sizeof(Entry) == 32, "entry is 32 bytes");

// Per-tree descriptor of a forest (a batch of independent trees, one per
// scene).  Offsets are in elements of the forest-wide arrays.
struct TreeDesc {
  int p0;     // first point of this tree in pts / x (and first row of seg)
  int n;      // number of support points
  int node0;  // first Entry of this tree in `nodes` (levels*cap*2 entries)
  int q0;     // first slot of this tree in `qorder` (sum of level sizes)
  int cap;    // stored internal nodes: the kept radix-tree nodes (those over
              // more than `leaf` points) get compact indices below cap
};

// Compact-node capacity of a tree of n points with leaves of at most `leaf`
// points.  A kept node has two children and the leaf records partition the
// points, so kept = records - 1 < 3n/leaf whenever the records average more
// than leaf/3 points (and always for leaf <= 3); measured on rooms, clustered
// scenes with duplicates and uniform clouds the kept count is 0.66-0.80 of
// 2n/leaf + 64.  A tree whose kept nodes exceed cap is flagged at build time
// and its queries take the exact scan.  GSA_NODE_CAP_LIMIT (a test build)
// caps it further so that the overflow path runs.
#ifndef GSA_NODE_CAP_LIMIT
#define GSA_NODE_CAP_LIMIT 0x7fffffff
#endif
__host__ __device__ inline int node_capacity(int n, int leaf) {
  long long c = 3ll * ((n + (long long)leaf - 1) / leaf) + 64;
  const long long m = n > 1 ? n - 1 : 1;
  if (c > m) c = m;
  if (c > GSA_NODE_CAP_LIMIT) c = GSA_NODE_CAP_LIMIT;
  return (int)(c < 1 ? 1 : c);
}

struct ForestView {
  const TreeDesc* desc;
  const float4* pts;    // leaf order; within a leaf ascending ID; w = ID bits
  const float4* lpts;   // [tree][level 1..][m_l] members of level l, leaf order
  const Entry* nodes;   // [tree][level][node][2]
  const Entry* root;    // [tree][level]
  const int* qorder;    // [tree][level][m_l] original IDs < m_l in leaf order
  const int* wrank;     // [point][level] members of the level before the
                        // point's leaf-order position
  const int* cut;       // [tree][level][kCutStride]: count, then up to kCutMax
                        // entry indices (-1: the root) that cover the tree
  const int* ovf;       // [tree]: 1 when the kept nodes exceeded the tree's
                        // capacity (the tree is unusable: exact scans)
  const float* x;       // borrowed original coordinates (AoS, 3 floats)
  int levels;           // 4 for prefix trees, 1 otherwise
};

__host__ __device__ inline int level_size(int n, int level) {
  return level <= 0 ? n : (n >> (2 * level));
}

// Leaf-ordered points of one tree's level: `pts` for level 0, else the
// level's member array (a tree's levels 1.. follow one another in `lpts`,
// starting at q0 - p0, the member count of the earlier trees' levels 1..).
__device__ inline const float4* level_pts(const ForestView& f,
                                          const TreeDesc& d, int level) {
  if (level <= 0) return f.pts + d.p0;
  size_t o = (size_t)(d.q0 - d.p0);
  for (int k = 1; k < level; ++k) o += level_size(d.n, k);
  return f.lpts + o;
}

__device__ inline int leaf_ref(int start, int count) {
  return ~((start << 5) | (count - 1));
}
__device__ inline void leaf_decode(int ref, int& start, int& count) {
  int v = ~ref;
  start = v >> 5;
  count = (v & 31) + 1;
}
// A level leaf with no member of its level (start 2^26 - 1 with 32 points,
// which no tree of at most kMaxPoints points has).  Its box is empty, so no
// query enters it; the builder reads its member count as 0.
constexpr int kEmptyLeaf = INT_MIN;
__device__ inline int level_leaf_count(int ref) {
  if (ref == kEmptyLeaf) return 0;
  return (~ref & 31) + 1;
}

__device__ inline Entry load_entry(const Entry* e) {
  const float4* p = reinterpret_cast<const float4*>(e);
  float4 a = __ldg(p), b = __ldg(p + 1);
  Entry r;
  r.lox = a.x; r.loy = a.y; r.loz = a.z; r.minid = __float_as_int(a.w);
  r.hix = b.x; r.hiy = b.y; r.hiz = b.z; r.ref = __float_as_int(b.w);
  return r;
}

__device__ inline void store_entry(Entry* e, const Entry& r) {
  float4* p = reinterpret_cast<float4*>(e);
  p[0] = make_float4(r.lox, r.loy, r.loz, __int_as_float(r.minid));
  p[1] = make_float4(r.hix, r.hiy, r.hiz, __int_as_float(r.ref));
}

// Exact squared distance ((dx*dx + dy*dy) + dz*dz), every operation rounded
// to nearest, never contracted into FMA, subnormals kept (GSA
// csrc/gsa_bvh.cu:278-281, csrc/reference_queries.cu:34-35, docs/api.md).
__device__ __forceinline__ float exact_d2(float qx, float qy, float qz,
                                          float px, float py, float pz) {
  float dx = __fsub_rn(qx, px), dy = __fsub_rn(qy, py), dz = __fsub_rn(qz, pz);
  return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)),
                   __fmul_rn(dz, dz));
}

// Squared point-to-box distance rounded toward -inf at every step, so it never
// exceeds exact_d2 of any point inside the box (GSA csrc/gsa_bvh.cu:121-132).
// An empty box (lo > hi) is reported as +inf.
__device__ __forceinline__ float lower_d2(float qx, float qy, float qz,
                                         const Entry& b) {
  if (b.lox > b.hix) return __int_as_float(0x7f800000);
  float dx = fmaxf(0.f, fmaxf(__fsub_rd(b.lox, qx), __fsub_rd(qx, b.hix)));
  float dy = fmaxf(0.f, fmaxf(__fsub_rd(b.loy, qy), __fsub_rd(qy, b.hiy)));
  float dz = fmaxf(0.f, fmaxf(__fsub_rd(b.loz, qz), __fsub_rd(qz, b.hiz)));
  return __fadd_rd(__fadd_rd(__fmul_rd(dx, dx), __fmul_rd(dy, dy)),
                   __fmul_rd(dz, dz));
}

// Squared box-to-box distance rounded toward -inf at every step.  Each
// round-down difference is monotone in its arguments, so for every point q of
// the box [l, h] the result is at most lower_d2(q, b): a node that fails a
// test against it holds no point within the radius of any such q.
__device__ __forceinline__ float box_lower_d2(float lx, float ly, float lz,
                                             float hx, float hy, float hz,
                                             const Entry& b) {
  if (b.lox > b.hix) return __int_as_float(0x7f800000);
  float dx = fmaxf(0.f, fmaxf(__fsub_rd(b.lox, hx), __fsub_rd(lx, b.hix)));
  float dy = fmaxf(0.f, fmaxf(__fsub_rd(b.loy, hy), __fsub_rd(ly, b.hiy)));
  float dz = fmaxf(0.f, fmaxf(__fsub_rd(b.loz, hz), __fsub_rd(lz, b.hiz)));
  return __fadd_rd(__fadd_rd(__fmul_rd(dx, dx), __fmul_rd(dy, dy)),
                   __fmul_rd(dz, dz));
}

__device__ __forceinline__ bool finite3(float a, float b, float c) {
  return isfinite(a) && isfinite(b) && isfinite(c);
}

// Order-preserving unsigned key of a float (finite and infinite values) and
// its inverse, for integer min/max reductions of coordinates.
__device__ __forceinline__ unsigned float_key(float f) {
  unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(unsigned k) {
  unsigned u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

}  // namespace gsa
