// SPDX-License-Identifier: Apache-2.0
// Exact ordered radius query and exact 3NN query over a prefix-bounds forest.
//
// Semantics follow GSA csrc/gsa_bvh.cu:282-343 (radius_ordered) and
// csrc/gsa_bvh.cu:149-211 (query3): the first `ns` qualifying support IDs
// < m in ascending ID order with d2 < r*r (pad with the first, zero row when
// none); the three smallest finite squared distances in (d2, id) order,
// missing entries (inf, 0).  Results do not depend on traversal order.
//
// Execution model (B200): one warp serves a packet of 32 queries at once (16
// or 8 when a launch would not fill the SMs, see packet_width).  Queries are
// visited in the tree's leaf order (for a query array that is a prefix of the
// support, neighbouring lanes hold neighbouring points), so the lanes need
// nearly the same part of the tree.  Three forms:
//   * packet-frontier kernels (default for the tree): the tree is culled once
//     against the box of the warp's queries, starting from the level's cut of
//     up to 32 entries, 32 child entries per step, and the surviving leaves
//     are processed as dense (query x point) pairs;
//   * per-query packet walks (walk_ordered, walk_knn3): one query per lane,
//     a node entered when any lane needs it, node entries and leaf points
//     loaded once per warp as 16-byte broadcast loads; the radius walk visits
//     children in ascending minimum-ID order so the reference's "K found and
//     minid >= K-th ID" early exit applies.  They answer what the frontier
//     kernels hand back (more than 32 radius hits when a lane holds
//     thousands, no finite 3NN bound, frontier overflow) and run alone in a
//     test variant; radius lanes with 33-256 hits take dense_walk, a
//     frontier over their box whose leaves are entered in minimum-ID order;
//   * warp scans of the support in original order, for small prefixes.
// A walk's stack overflow (impossible for STACK >= 97 on a Karras tree of
// 64-bit keys) falls back to the exact original-order scan and is counted,
// as in the reference.
#include <atomic>
#include <algorithm>
#include "forest.cuh"
#include "pool.cuh"

#ifndef GSA_STACK
#define GSA_STACK 128
#endif
// Support prefixes up to these sizes are answered by the warp scans below
// instead of a tree walk (same results).  Timed on the room hierarchy: a
// 375-point radius prefix scans in 27 us against 48 us for the frontier
// kernel, a 1500-point one takes 175 us against 64 us; a 375-point 3NN prefix
// 135 us against 64 us.
#ifndef GSA_RADIUS_SCAN_MAX
#define GSA_RADIUS_SCAN_MAX 512
#endif
#ifndef GSA_KNN_SCAN_MAX
#define GSA_KNN_SCAN_MAX 128
#endif
// Tree-walk radius kernel: 1 culls with the warp's packet box and processes
// leaves as dense (query, point) pairs (radius_frontier_kernel); 0 is the
// ordered per-query packet walk (radius_kernel) throughout.
#ifndef GSA_RADIUS_FRONTIER
#define GSA_RADIUS_FRONTIER 1
#endif
// Tree-walk 3NN kernel: 1 collects candidates within a per-query window bound
// (knn3_frontier_kernel); 0 is the nearest-first per-query walk (knn3_kernel).
#ifndef GSA_KNN_FRONTIER
#define GSA_KNN_FRONTIER 1
#endif

namespace gsa {
namespace {

constexpr int kQThreads = 256;
constexpr int kQWarps = kQThreads / 32;

struct QArgs {
  ForestView f;
  const float* q;
  const int* qstart;  // per-tree first input query row (device) or null
  const int* qseg;    // per-tree output row offsets (device) or null
  int nq;             // single tree: number of queries
  int m;              // support prefix for every tree; 0 = level size
  int level;        // bounds level, -1 = all points (level 0 data)
  float radius;
  int ns;
  int* out;
  float* dout;
  int* fallback;
  int pw;             // frontier kernels: queries per warp (8, 16 or 32)
  const int* qperm;   // single tree: query rows in a spatial (Morton) order,
                      // walked instead of the support's leaf order; null:
                      // the queries are taken to be the support's points
};

__device__ __forceinline__ bool nonempty(const Entry& e) {
  return e.lox <= e.hix;
}

// Largest stored level whose prefix still holds all Q queries.
__device__ __forceinline__ int query_level(int n, int levels, int Q) {
  int l = 0;
  while (l + 1 < levels && level_size(n, l + 1) >= Q) ++l;
  return l;
}

__device__ __forceinline__ int level_offset(int n, int l) {
  int o = 0;
  for (int k = 0; k < l; ++k) o += level_size(n, k);
  return o;
}

struct Slot {
  int qbase, qin, Q, m, slots, lev;
  const int* order;  // slot -> query (null: identity)
  bool ovf;          // the tree overflowed its node capacity: exact scans
  bool perm;         // order is a permutation of the Q query rows
};

__device__ __forceinline__ Slot slot_setup(const QArgs& a, const TreeDesc& d,
                                           int b) {
  Slot s;
  s.qbase = a.qseg ? a.qseg[b] : 0;
  s.qin = a.qstart ? a.qstart[b] : s.qbase;
  s.Q = a.qseg ? a.qseg[b + 1] - s.qbase : a.nq;
  s.m = a.m > 0 ? a.m : level_size(d.n, a.level);
  s.lev = a.level < 0 ? 0 : a.level;
  s.ovf = a.f.ovf[b] != 0;
  s.perm = a.qperm != nullptr;
  if (s.perm) {  // single tree: every query row once, in the given order
    s.slots = s.Q;
    s.order = a.qperm;
    return s;
  }
  int ql = s.Q <= d.n ? query_level(d.n, a.f.levels, s.Q) : 0;
  s.slots = s.Q <= d.n ? level_size(d.n, ql) : s.Q;
  s.order = a.f.qorder + d.q0 + level_offset(d.n, ql);
  if (s.ovf) s.order = nullptr;  // the build wrote no query order
  return s;
}

__device__ __forceinline__ int slot_query(const Slot& s, const TreeDesc& d,
                                          int t) {
  if (t >= s.slots) return -1;
  int qi = s.order && (s.perm || t < d.n) ? __ldg(s.order + t) : t;
  return qi < s.Q ? qi : -1;
}

__device__ __forceinline__ bool radius_test(const Entry& e, float px, float py,
                                            float pz, int m, int bound,
                                            float r2) {
  return e.minid < m && e.minid < bound && nonempty(e) &&
         lower_d2(px, py, pz, e) < r2;
}

struct RadiusCtx {
  const Entry* nodes;
  const Entry* root;
  const float4* pts;  // the bounds level's leaf-ordered points
  const float* xs;
  int m, K;
  float r2;
  long long max_steps;
  bool sorted;  // leaf IDs ascend (level 0 leaves)
};

// Ordered packet walk for the active lanes: one warp, one query per lane,
// children visited in ascending minimum-ID order, per-lane first-K list L
// kept sorted (insertion), "K found and minid >= K-th ID" prunes subtrees.
// `bound0` (per lane) is an exclusive bound known to hold the first K IDs
// (INT_MAX when none is known).  Returns the lane's count; sets overflow
// (warp-uniform) on stack overflow.
template <int STACK>
__device__ int walk_ordered(const RadiusCtx& c, bool active, float px,
                            float py, float pz, int* L, int* stk,
                            bool& overflow, int bound0 = INT_MAX) {
  const int K = c.K, m = c.m;
  const float r2 = c.r2;
  int count = 0, bound = bound0;
  Entry cur = load_entry(c.root);
  bool need = active && radius_test(cur, px, py, pz, m, bound, r2);
  int top = 0;
  // A valid tree is visited at most once per node; the cap only guards
  // against a corrupted handle (then the exact scan answers).
  long long steps = 0;
  while (true) {
    if (++steps > c.max_steps) {
      overflow = true;
      break;
    }
    if (!__any_sync(kFull, need)) {
      if (top == 0) break;
      int ei = stk[--top];
      cur = load_entry(c.nodes + ei);
      need = active && radius_test(cur, px, py, pz, m, bound, r2);
      continue;
    }
    if (cur.ref >= 0) {
      const Entry* ch = c.nodes + (size_t)cur.ref * 2;
      Entry c0 = load_entry(ch), c1 = load_entry(ch + 1);
      bool n0 = need && radius_test(c0, px, py, pz, m, bound, r2);
      bool n1 = need && radius_test(c1, px, py, pz, m, bound, r2);
      bool a0 = __any_sync(kFull, n0), a1 = __any_sync(kFull, n1);
      if (a0) {
        if (a1) {
          if (top == STACK) {
            overflow = true;
            break;
          }
          stk[top++] = cur.ref * 2 + 1;
        }
        cur = c0;
        need = n0;
      } else {
        cur = c1;
        need = n1;
      }
    } else {
      int start, cnt;
      leaf_decode(cur.ref, start, cnt);
      for (int j = 0; j < cnt; ++j) {
        float4 pt = __ldg(c.pts + start + j);
        int id = __float_as_int(pt.w);
        bool cand = need && id < m && id < bound;
        // in an ascending leaf no later point can qualify
        if (c.sorted && !__any_sync(kFull, cand)) break;
        if (cand && exact_d2(px, py, pz, pt.x, pt.y, pt.z) < r2) {
          int pos = count < K ? count : K - 1;
          while (pos > 0 && L[pos - 1] > id) {
            L[pos] = L[pos - 1];
            --pos;
          }
          L[pos] = id;
          if (count < K) ++count;
          if (count == K) bound = L[K - 1];
        }
      }
      need = false;
    }
  }
  return count;
}

// Exact original-order scan of one query (stack-overflow fallback).
__device__ int scan_ordered(const RadiusCtx& c, float px, float py, float pz,
                            int* L) {
  int count = 0;
  for (int id = 0; id < c.m && count < c.K; ++id) {
    const float* p = c.xs + 3ll * id;
    if (exact_d2(px, py, pz, p[0], p[1], p[2]) < c.r2) L[count++] = id;
  }
  return count;
}

// Row of each lane's query: K IDs, padded with the first, zero when none;
// written cooperatively, one coalesced row per step.
__device__ void write_rows(int* out, const int* lists_w, int stride, int qi,
                           int count, int qbase, int K, int lane) {
  __syncwarp();
  for (int j = 0; j < 32; ++j) {
    int qj = __shfl_sync(kFull, qi, j);
    int cj = __shfl_sync(kFull, count, j);
    if (qj < 0) continue;
    if (lane < K) {
      const int* row = lists_w + j * stride;
      out[(size_t)(qbase + qj) * K + lane] = cj ? row[lane < cj ? lane : 0] : 0;
    }
  }
}

// As write_rows with 16-byte stores, four rows per step (K/4 lanes per row),
// when K is a multiple of 4 and `out` 16-byte aligned (then every row is);
// otherwise write_rows.
__device__ void write_rows4(int* out, const int* lists_w, int stride, int qi,
                            int count, int qbase, int K, int lane) {
  if ((K & 3) || (reinterpret_cast<uintptr_t>(out) & 15)) {
    write_rows(out, lists_w, stride, qi, count, qbase, K, lane);
    return;
  }
  __syncwarp();
  const int per = K >> 2;            // lanes per row
  const int rows = 32 / per;         // rows per step (4 at K = 32)
  const int r = lane / per, c = (lane - r * per) * 4;
  for (int j0 = 0; j0 < 32; j0 += rows) {
    const int j = j0 + r;
    const bool on = r < rows && j < 32;
    const int qj = __shfl_sync(kFull, qi, on ? j : 0);
    const int cj = __shfl_sync(kFull, count, on ? j : 0);
    if (!on || qj < 0) continue;
    const int* row = lists_w + j * stride;
    const int first = cj ? row[0] : 0;
    int4 v;
    v.x = c < cj ? row[c] : first;
    v.y = c + 1 < cj ? row[c + 1] : first;
    v.z = c + 2 < cj ? row[c + 2] : first;
    v.w = c + 3 < cj ? row[c + 3] : first;
    *reinterpret_cast<int4*>(out + (size_t)(qbase + qj) * K + c) = v;
  }
}

__device__ __forceinline__ RadiusCtx radius_ctx(const QArgs& a,
                                                const TreeDesc& d, int b,
                                                const Slot& s) {
  RadiusCtx c;
  c.nodes = a.f.nodes + d.node0 + (size_t)s.lev * d.cap * 2;
  c.root = a.f.root + b * a.f.levels + s.lev;
  c.pts = level_pts(a.f, d, s.lev);
  c.xs = a.f.x + 3ll * d.p0;
  c.m = s.m;
  c.K = a.ns;
  c.r2 = __fmul_rn(a.radius, a.radius);
  c.max_steps = 4ll * d.n + 64;
  c.sorted = s.lev == 0;
  return c;
}

template <int STACK>
__global__ void __launch_bounds__(kQThreads)
    radius_kernel(QArgs a) {
  __shared__ int lists[kQWarps][32][33];
  __shared__ int stack[kQWarps][STACK];
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  Slot s = slot_setup(a, d, b);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long t0 = ((long long)blockIdx.x * kQWarps + warp) * 32;
  if (t0 >= s.slots) return;  // warp-uniform
  int qi = slot_query(s, d, (int)t0 + lane);
  bool active = qi >= 0;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (active) {
    const float* qp = a.q + 3ll * (s.qin + qi);
    px = qp[0];
    py = qp[1];
    pz = qp[2];
  }
  RadiusCtx c = radius_ctx(a, d, b, s);
  int* L = lists[warp][lane];
  if (s.ovf) {  // tree-uniform: no usable tree, every query scans
    int count = 0;
    if (active) {
      atomicAdd(a.fallback, 1);
      count = scan_ordered(c, px, py, pz, L);
    }
    write_rows4(a.out, &lists[warp][0][0], 33, qi, count, s.qbase, c.K, lane);
    return;
  }
  bool overflow = false;
  int count = walk_ordered<STACK>(c, active, px, py, pz, L, stack[warp], overflow);
  if (overflow && active) {
    atomicAdd(a.fallback, 1);
    count = scan_ordered(c, px, py, pz, L);
  }
  write_rows4(a.out, &lists[warp][0][0], 33, qi, count, s.qbase, c.K, lane);
}

__device__ __forceinline__ void insert3(float v, int id, float& d0, float& d1,
                                        float& d2, int& i0, int& i1, int& i2) {
  if (!isfinite(v)) return;
  if (v < d2 || (v == d2 && id < i2)) {
    if (v < d1 || (v == d1 && id < i1)) {
      d2 = d1;
      i2 = i1;
      if (v < d0 || (v == d0 && id < i0)) {
        d1 = d0;
        i1 = i0;
        d0 = v;
        i0 = id;
      } else {
        d1 = v;
        i1 = id;
      }
    } else {
      d2 = v;
      i2 = id;
    }
  }
}

// The three best (d2, id) of a query, in order; (inf, INT_MAX) when missing.
struct Top3 {
  float d0, d1, d2;
  int i0, i1, i2;
};

__device__ __forceinline__ Top3 empty_top3() {
  const float inf = __int_as_float(0x7f800000);
  return Top3{inf, inf, inf, INT_MAX, INT_MAX, INT_MAX};
}

struct KnnCtx {
  const Entry* nodes;
  const Entry* root;
  const float4* pts;  // the bounds level's leaf-ordered points
  const float* xs;
  int m;
  long long max_steps;
  bool sorted;  // leaf IDs ascend (level 0 leaves)
};

__device__ __forceinline__ KnnCtx knn_ctx(const QArgs& a, const TreeDesc& d,
                                          int b, const Slot& s) {
  KnnCtx c;
  c.nodes = a.f.nodes + d.node0 + (size_t)s.lev * d.cap * 2;
  c.root = a.f.root + b * a.f.levels + s.lev;
  c.pts = level_pts(a.f, d, s.lev);
  c.xs = a.f.x + 3ll * d.p0;
  c.m = s.m;
  c.max_steps = 4ll * d.n + 64;
  c.sorted = s.lev == 0;
  return c;
}

// Nearest-first packet walk for the active lanes (one query per lane): the
// children a lane needs are visited in the order most needing lanes prefer,
// subtrees with a lower bound above the lane's third distance are skipped.
// Returns true (warp-uniform) on stack overflow or a step cap.
template <int STACK>
__device__ bool walk_knn3(const KnnCtx& c, bool active, float px, float py,
                          float pz, Top3& t, int* stk) {
  const int m = c.m;
  Entry cur = load_entry(c.root);
  bool need = active && cur.minid < m && nonempty(cur) &&
              lower_d2(px, py, pz, cur) <= t.d2;
  int top = 0;
  long long steps = 0;
  while (true) {
    if (++steps > c.max_steps) return true;
    if (!__any_sync(kFull, need)) {
      if (top == 0) return false;
      int ei = stk[--top];
      cur = load_entry(c.nodes + ei);
      need = active && cur.minid < m && nonempty(cur) &&
             lower_d2(px, py, pz, cur) <= t.d2;
      continue;
    }
    if (cur.ref >= 0) {
      const Entry* ch = c.nodes + (size_t)cur.ref * 2;
      Entry c0 = load_entry(ch), c1 = load_entry(ch + 1);
      float l0 = lower_d2(px, py, pz, c0), l1 = lower_d2(px, py, pz, c1);
      bool n0 = need && c0.minid < m && nonempty(c0) && l0 <= t.d2;
      bool n1 = need && c1.minid < m && nonempty(c1) && l1 <= t.d2;
      unsigned b0 = __ballot_sync(kFull, n0), b1 = __ballot_sync(kFull, n1);
      if (b0 && b1) {
        unsigned both = b0 & b1;
        unsigned pref1 = __ballot_sync(kFull, n0 && n1 && l1 < l0);
        bool first1 = 2 * __popc(pref1) > __popc(both);
        if (top == STACK) return true;
        stk[top++] = cur.ref * 2 + (first1 ? 0 : 1);
        cur = first1 ? c1 : c0;
        need = first1 ? n1 : n0;
      } else if (b0) {
        cur = c0;
        need = n0;
      } else {
        cur = c1;
        need = n1;
      }
    } else {
      int start, cnt;
      leaf_decode(cur.ref, start, cnt);
      for (int j = 0; j < cnt; ++j) {
        float4 pt = __ldg(c.pts + start + j);
        int id = __float_as_int(pt.w);
        if (id >= m) {
          if (c.sorted) break;
          continue;
        }
        if (need)
          insert3(exact_d2(px, py, pz, pt.x, pt.y, pt.z), id, t.d0, t.d1, t.d2,
                  t.i0, t.i1, t.i2);
      }
      need = false;
    }
  }
}

// Exact original-order scan of one query (stack-overflow fallback).
__device__ Top3 scan_knn3(const KnnCtx& c, float px, float py, float pz) {
  Top3 t = empty_top3();
  for (int id = 0; id < c.m; ++id) {
    const float* p = c.xs + 3ll * id;
    insert3(exact_d2(px, py, pz, p[0], p[1], p[2]), id, t.d0, t.d1, t.d2, t.i0,
            t.i1, t.i2);
  }
  return t;
}

__device__ __forceinline__ void write_top3(const QArgs& a, const Slot& s,
                                           int qi, const Top3& t) {
  size_t o = (size_t)(s.qbase + qi) * 3;
  a.dout[o] = t.d0;
  a.dout[o + 1] = t.d1;
  a.dout[o + 2] = t.d2;
  a.out[o] = t.i0 == INT_MAX ? 0 : t.i0;
  a.out[o + 1] = t.i1 == INT_MAX ? 0 : t.i1;
  a.out[o + 2] = t.i2 == INT_MAX ? 0 : t.i2;
}

template <int STACK>
__global__ void __launch_bounds__(kQThreads)
    knn3_kernel(QArgs a) {
  __shared__ int stack[kQWarps][STACK];
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  Slot s = slot_setup(a, d, b);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long t0 = ((long long)blockIdx.x * kQWarps + warp) * 32;
  if (t0 >= s.slots) return;
  int qi = slot_query(s, d, (int)t0 + lane);
  bool active = qi >= 0;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (active) {
    const float* qp = a.q + 3ll * (s.qin + qi);
    px = qp[0];
    py = qp[1];
    pz = qp[2];
  }
  KnnCtx c = knn_ctx(a, d, b, s);
  if (s.ovf) {  // tree-uniform: no usable tree, every query scans
    if (active) {
      atomicAdd(a.fallback, 1);
      write_top3(a, s, qi, scan_knn3(c, px, py, pz));
    }
    return;
  }
  Top3 t = empty_top3();
  bool overflow = walk_knn3<STACK>(c, active, px, py, pz, t, stack[warp]);
  if (overflow && active) {
    atomicAdd(a.fallback, 1);
    t = scan_knn3(c, px, py, pz);
  }
  if (active) write_top3(a, s, qi, t);
}

// ---------------------------------------------------------------------------
// Packet-frontier kernels.  A warp's 32 queries are neighbours in leaf order,
// so the tree is culled once for all of them against the box of the warp's
// queries (box_lower_d2), 32 child entries per step (one per lane) from a
// warp frontier stack, instead of a per-query test of two children per step.
// Leaves that survive are queued and handled in batches of up to 32: one
// lane loads each queued leaf's entry (one round trip for the batch), every
// query tests every batch leaf's box from shuffled registers, and the leaves
// some query needs are processed as (query x point) pairs, the leaf's points
// held one per lane (w = count rounded up to a power of two, 32/w queries
// per step), with the next leaf's points already loading.  A hit is ranked
// by ballot into a per-query shared buffer.
//
// Radius (KNN = false): every query's bound is r*r, a hit is d2 < r*r, the
// buffer holds IDs; more than kPacketCap hits, or a frontier overflow, sends
// the query to the ordered walk.  3NN (KNN = true): the bound B of a query
// starts as the third distance within a window of the level's members around
// its own member rank, a hit is d2 <= B and the buffer holds point positions;
// a buffer that could overflow is first cut to its best three (lowering B).
// Every point of the final answer satisfies the hit test at every moment, so
// both answers are exact.
// Warps (packets) per frontier block.  Two rather than four: a block's
// slot is freed when its slowest packet ends, so smaller blocks waste less
// of an SM on finished warps (64 scenes: 3NN stage 0 436 -> 422 us, radius
// 592 -> 587 us; one warp per block hits the 32-block limit first).
#ifndef GSA_FRONTIER_WARPS
#define GSA_FRONTIER_WARPS 2
#endif
constexpr int kFWarps = GSA_FRONTIER_WARPS;
constexpr int kPacketCap = 32;  // radius hits per query; holds a K-list (K<=32)
constexpr int kCandCap = 35;    // 3NN candidates: three kept + a leaf of 32
constexpr int kWindow = 16;     // 3NN bound: 2*kWindow members (3NN stages
                                // 0-2 of the room hierarchy with 8 / 12 / 16 /
                                // 24 / 32 members: 860 / 789 / 768 / 754 /
                                // 736 us)

// Box of the warp's packet queries and the node-test bound (r*r or the
// largest B of the packet).
struct Packet {
  float lx, ly, lz, hx, hy, hz, R2;
};

__device__ __forceinline__ Packet make_packet(bool in, float px, float py,
                                              float pz, float b) {
  Packet p;
  p.lx = key_float(__reduce_min_sync(kFull, in ? float_key(px) : ~0u));
  p.ly = key_float(__reduce_min_sync(kFull, in ? float_key(py) : ~0u));
  p.lz = key_float(__reduce_min_sync(kFull, in ? float_key(pz) : ~0u));
  p.hx = key_float(__reduce_max_sync(kFull, in ? float_key(px) : 0u));
  p.hy = key_float(__reduce_max_sync(kFull, in ? float_key(py) : 0u));
  p.hz = key_float(__reduce_max_sync(kFull, in ? float_key(pz) : 0u));
  p.R2 = key_float(__reduce_max_sync(kFull, in ? float_key(b) : 0u));
  return p;
}

template <bool KNN>
__device__ __forceinline__ bool within(float d2, float bound) {
  return KNN ? d2 <= bound : d2 < bound;
}

// One queued leaf's points for the pair steps: lane k*w + j holds point j.
struct LeafPts {
  float4 pt;
  int start, cnt, logw;
};

__device__ __forceinline__ LeafPts leaf_points(const float4* pts, int ref,
                                               int lane) {
  LeafPts L;
  leaf_decode(ref, L.start, L.cnt);
  L.logw = L.cnt <= 1 ? 0 : 32 - __clz(L.cnt - 1);
  int j = lane & ((1 << L.logw) - 1);
  L.pt = j < L.cnt ? __ldg(pts + L.start + j)
                   : make_float4(0.f, 0.f, 0.f, __int_as_float(INT_MAX));
  return L;
}

// Per-warp shared state of a frontier kernel.
template <int CAP, int FRONT>
struct WarpBufs {
  int buf[32][CAP + 1];  // per-query hits (IDs) or candidates (positions)
  float4 qa[32];         // pair steps: active query i's coordinates, and its
                         // lane (radius) or its bound (3NN) in w
  int amap[32];          // pair steps (3NN): active query i's lane
  int leafq[64];         // queued leaf entries (-1: the root)
  int front[FRONT];      // frontier stack of internal nodes
};

// Best three of a lane's candidate positions, kept at the row's front.
__device__ __forceinline__ Top3 cut_candidates(const float4* pts, int* row,
                                               int& nc, float px, float py,
                                               float pz) {
  Top3 t = empty_top3();
  int q0 = 0, q1 = 0, q2 = 0;
  for (int i = 0; i < nc; ++i) {
    int pos = row[i];
    float4 pt = __ldg(pts + pos);
    int id = __float_as_int(pt.w);
    float v = exact_d2(px, py, pz, pt.x, pt.y, pt.z);
    if (!isfinite(v)) continue;
    if (v < t.d2 || (v == t.d2 && id < t.i2)) {
      if (v < t.d1 || (v == t.d1 && id < t.i1)) {
        t.d2 = t.d1; t.i2 = t.i1; q2 = q1;
        if (v < t.d0 || (v == t.d0 && id < t.i0)) {
          t.d1 = t.d0; t.i1 = t.i0; q1 = q0;
          t.d0 = v; t.i0 = id; q0 = pos;
        } else {
          t.d1 = v; t.i1 = id; q1 = pos;
        }
      } else {
        t.d2 = v; t.i2 = id; q2 = pos;
      }
    }
  }
  nc = (t.i0 != INT_MAX) + (t.i1 != INT_MAX) + (t.i2 != INT_MAX);
  row[0] = q0;
  row[1] = q1;
  row[2] = q2;
  return t;
}

// One batch of queued leaves lq[0..nleaf) (see the section comment).  `in`:
// the lane's query takes part; `bound`: its current bound (r*r, the same on
// every lane, or B); `nc`: its buffer count.
template <bool KNN, int CAP, int FRONT>
__device__ void leaf_batches(WarpBufs<CAP, FRONT>& W, const Entry* nodes,
                             const Entry* root, const float4* pts, int nleaf,
                             int m, bool in, float px, float py, float pz,
                             float& bound, int& nc) {
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (int b0 = 0; b0 < nleaf; b0 += 32) {
    const int nb = min(32, nleaf - b0);
    Entry le;
    le.lox = le.loy = le.loz = 1.f;
    le.hix = le.hiy = le.hiz = 0.f;  // empty
    le.minid = INT_MAX;
    le.ref = -1;
    if (lane < nb) {
      int ei = W.leafq[b0 + lane];
      le = load_entry(ei >= 0 ? nodes + ei : root);
    }
    unsigned myM = 0;  // lane li: queries that need batch leaf li
    for (int li = 0; li < nb; ++li) {
      Entry e;
      e.lox = __shfl_sync(kFull, le.lox, li);
      e.loy = __shfl_sync(kFull, le.loy, li);
      e.loz = __shfl_sync(kFull, le.loz, li);
      e.hix = __shfl_sync(kFull, le.hix, li);
      e.hiy = __shfl_sync(kFull, le.hiy, li);
      e.hiz = __shfl_sync(kFull, le.hiz, li);
      bool need = in && within<KNN>(lower_d2(px, py, pz, e), bound);
      unsigned M = __ballot_sync(kFull, need);
      if (lane == li) myM = M;
    }
    unsigned act = __ballot_sync(kFull, myM != 0);
    if (!act) continue;
    int cur = __ffs(act) - 1;
    act &= act - 1;
    LeafPts L = leaf_points(pts, __shfl_sync(kFull, le.ref, cur), lane);
    while (true) {
      // start loading the next needed leaf's points
      const int nxt = act ? __ffs(act) - 1 : -1;
      if (act) act &= act - 1;
      const int nref = __shfl_sync(kFull, le.ref, nxt < 0 ? 0 : nxt);
      LeafPts Ln;
      if (nxt >= 0) Ln = leaf_points(pts, nref, lane);
      const unsigned M = __shfl_sync(kFull, myM, cur);
      const bool need = (M >> lane) & 1u;
      if (KNN && __any_sync(kFull, need && nc + L.cnt > CAP)) {
        if (need && nc + L.cnt > CAP) {
          Top3 t = cut_candidates(pts, W.buf[lane], nc, px, py, pz);
          if (nc == 3) bound = t.d2;
        }
      }
      const int nA = __popc(M);
      const int mine = __popc(M & lt);
      if (need) {
        W.qa[mine] = make_float4(px, py, pz, KNN ? bound : __int_as_float(lane));
        if (KNN) W.amap[mine] = lane;
      }
      __syncwarp();
      const int logw = L.logw;
      const int w = 1 << logw, per = 32 >> logw;
      const int k = lane >> logw, j = lane & (w - 1), kw = k << logw;
      const unsigned seg0 = w == 32 ? kFull : (1u << w) - 1u;
      const int id = __float_as_int(L.pt.w);
      const bool pv = j < L.cnt && id < m;
      for (int base = 0; base < nA; base += per) {
        const int idx = base + k;
        const bool valid = pv && idx < nA;
        // one 16-byte load per step: the query's coordinates with its lane
        // (radius; the bound r*r is the same for every query) or its bound
        const float4 qc = W.qa[idx < nA ? idx : 0];
        const bool hit = valid && within<KNN>(exact_d2(qc.x, qc.y, qc.z, L.pt.x,
                                                       L.pt.y, L.pt.z),
                                              KNN ? qc.w : bound);
        const unsigned hm = __ballot_sync(kFull, hit);
        if (!hm) continue;  // warp-uniform
        const int q = KNN ? W.amap[idx < nA ? idx : 0] : __float_as_int(qc.w);
        // hits of this query's segment below this lane, after its count
        const int slot = __shfl_sync(kFull, nc, q) + __popc((hm & lt) >> kw);
        if (hit && (KNN || slot < CAP)) W.buf[q][slot] = KNN ? L.start + j : id;
        const int mk = mine - base;
        if (need && (unsigned)mk < (unsigned)per)
          nc += __popc((hm >> (mk << logw)) & seg0);
      }
      __syncwarp();
      if (nxt < 0) break;
      cur = nxt;
      L = Ln;
    }
  }
}

// Frontier walk of the packet; leaves go through leaf_batches.  Returns
// true (warp-uniform) when the frontier would exceed its stack or the step
// cap is reached.  The walk starts from the level's cut (`cut`: count, then
// up to kCutMax entries that cover the tree; -1 is the root), tested in one
// step.  Queued leaves are processed before a round once 32 are waiting, so
// the queue (64) holds the cut's leaves or one round's on top of fewer than
// 32.
template <bool KNN, int CAP, int FRONT>
__device__ bool frontier_walk(WarpBufs<CAP, FRONT>& W, const Entry* nodes,
                              const Entry* root, const int* cut,
                              const float4* pts, long long max_steps, int m,
                              const Packet& pk, bool in, float px, float py,
                              float pz, float& bound, int& nc) {
  static_assert(kCutMax <= 64, "the leaf queue holds the whole cut");
  constexpr int CH = kCutMax / 32;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  int top = 0, nleaf = 0;
  {
    const int ncut = cut[0];
    Entry e[CH];
    int ei[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      ei[c] = -1;
      if (c * 32 + lane < ncut) {
        ei[c] = cut[1 + c * 32 + lane];
        e[c] = load_entry(ei[c] >= 0 ? nodes + ei[c] : root);
      }
    }
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      bool pass = false, inner = false;
      if (c * 32 + lane < ncut) {
        pass = e[c].minid < m &&
               within<KNN>(box_lower_d2(pk.lx, pk.ly, pk.lz, pk.hx, pk.hy,
                                        pk.hz, e[c]),
                           pk.R2);
        inner = e[c].ref >= 0;
      }
      unsigned bi = __ballot_sync(kFull, pass && inner);
      unsigned bl = __ballot_sync(kFull, pass && !inner);
      if (top + __popc(bi) > FRONT) return true;
      if (pass && inner) W.front[top + __popc(bi & lt)] = e[c].ref;
      if (pass && !inner) W.leafq[nleaf + __popc(bl & lt)] = ei[c];
      top += __popc(bi);
      nleaf += __popc(bl);
    }
  }
  __syncwarp();
  long long steps = 0;
  while (top > 0 || nleaf > 0) {
    if (++steps > max_steps) return true;
    if (nleaf >= 32 || top == 0) {
      leaf_batches<KNN>(W, nodes, root, pts, nleaf, m, in, px, py, pz, bound,
                        nc);
      nleaf = 0;
      __syncwarp();
      continue;
    }
    // Pop up to 16 internal nodes; lane 2i+j tests child j of node i.
    int P = min(top, 16);
    bool pass = false, inner = false;
    int ei = 0, ref = 0;
    if (lane < 2 * P) {
      ei = 2 * W.front[top - P + (lane >> 1)] + (lane & 1);
      Entry e = load_entry(nodes + ei);
      pass = e.minid < m &&
             within<KNN>(box_lower_d2(pk.lx, pk.ly, pk.lz, pk.hx, pk.hy,
                                      pk.hz, e),
                         pk.R2);
      inner = e.ref >= 0;
      ref = e.ref;
    }
    __syncwarp();
    top -= P;
    unsigned bi = __ballot_sync(kFull, pass && inner);
    unsigned bl = __ballot_sync(kFull, pass && !inner);
    int ni = __popc(bi);
    if (top + ni > FRONT) return true;
    if (pass && inner) W.front[top + __popc(bi & lt)] = ref;
    if (pass && !inner) W.leafq[nleaf + __popc(bl & lt)] = ei;
    top += ni;
    nleaf += __popc(bl);
    __syncwarp();
  }
  return false;
}

// Sorts h[0..count) ascending (count <= N <= W, W a power of two) with a
// bitonic network over registers in its all-ascending form (each merge
// starts with a flip step i <-> i ^ (k-1), then half-cleaners; every
// comparator puts the minimum at the lower index).  Slots from count on hold
// INT_MAX, so slots N..W-1 would stay INT_MAX throughout and every
// comparator touching them is dropped at compile time: W = 32 costs 240
// comparators at N = 32, 168 at 24, 134 at 20; W = 16, N = 16 costs 80.
template <int W, int N>
__device__ __forceinline__ void sort_hits(int* h, int count) {
  int v[W];
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] = i < N && i < count ? h[i] : INT_MAX;
#pragma unroll
  for (int k = 2; k <= W; k <<= 1) {
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const int l = i ^ (k - 1);
      if (l > i && l < N) {
        const int lo = min(v[i], v[l]), hi = max(v[i], v[l]);
        v[i] = lo;
        v[l] = hi;
      }
    }
#pragma unroll
    for (int j = k >> 2; j > 0; j >>= 1) {
#pragma unroll
      for (int i = 0; i < W; ++i) {
        const int l = i ^ j;
        if (l > i && l < N) {
          const int lo = min(v[i], v[l]), hi = max(v[i], v[l]);
          v[i] = lo;
          v[l] = hi;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < count) h[i] = v[i];
}

#ifndef GSA_DENSE_WALK
#define GSA_DENSE_WALK 1
#endif
// Largest hit count of a spilled lane up to which dense_walk answers the
// packet's spilled lanes; above it they take the ordered walk, whose
// depth-first descent in minimum-ID order finds the first K of thousands of
// hits (a packet inside a cluster that r covers whole) with less work.
#ifndef GSA_DENSE_MAX_HITS
#define GSA_DENSE_MAX_HITS 256
#endif

// Ascending sort of one key per lane across the warp (bitonic network over
// lanes); `src` travels with its key.
__device__ __forceinline__ void warp_sort_keys(int& key, int& src) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int ok = __shfl_xor_sync(kFull, key, j);
      const int os = __shfl_xor_sync(kFull, src, j);
      const bool up = (lane & k) == 0, lower = (lane & j) == 0;
      // the lower lane of an ascending pair keeps the smaller key
      const bool take = (ok < key || (ok == key && os < src)) == (lower == up);
      if (take) {
        key = ok;
        src = os;
      }
    }
  }
}

// Dense neighbourhoods: lanes with more than kPacketCap hits inside r (the
// spilled lanes of a packet) need the first K IDs among all of them.  They
// walk the tree together as a frontier over the box of their queries (as
// frontier_walk), pruning every node whose minimum ID reaches the warp's
// bound, the largest of the lanes' bounds (a lane's bound: its K-th ID once
// it holds K, else b0, an ID above its first K known from the frontier
// pass).  Each batch of queued leaves is sorted by minimum ID and entered in
// that order, every lane inserting the leaf's points inside r with ID below
// its bound into its ascending first-K list (as walk_ordered), until a
// leaf's minimum ID reaches the warp's bound.  The ordered walk enters the
// same subtrees one dependent step at a time; here a step tests up to 32
// child entries and the bounds fall as soon as the smallest-ID leaves are
// in.  Returns the lane's count; sets `overflow` (warp-uniform) when the
// frontier outgrows its stack or the step cap, for walk_ordered to answer.
template <int FRONT>
__device__ __forceinline__ int dense_walk(WarpBufs<kPacketCap, FRONT>& W,
                                       RadiusCtx c, const int* cut, bool act,
                                       float px, float py, float pz, int b0,
                                       bool& overflow) {
  constexpr int CH = kCutMax / 32;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  const int K = c.K, m = c.m;
  const float r2 = c.r2;
  int* L = W.buf[lane];
  int count = 0, bound = act ? b0 : 0;
  int wb = (int)__reduce_max_sync(kFull, (unsigned)bound);
  const Packet pk = make_packet(act, px, py, pz, r2);
  overflow = false;
  int top = 0, nleaf = 0;
  {
    const int ncut = cut[0];
    Entry e[CH];
    int ei[CH];
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      ei[k] = -1;
      if (k * 32 + lane < ncut) {
        ei[k] = cut[1 + k * 32 + lane];
        e[k] = load_entry(ei[k] >= 0 ? c.nodes + ei[k] : c.root);
      }
    }
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      bool pass = false, inner = false;
      if (k * 32 + lane < ncut) {
        pass = e[k].minid < m && e[k].minid < wb &&
               box_lower_d2(pk.lx, pk.ly, pk.lz, pk.hx, pk.hy, pk.hz, e[k]) <
                   r2;
        inner = e[k].ref >= 0;
      }
      const unsigned bi = __ballot_sync(kFull, pass && inner);
      const unsigned bl = __ballot_sync(kFull, pass && !inner);
      if (top + __popc(bi) > FRONT) {
        overflow = true;
        return 0;
      }
      if (pass && inner) W.front[top + __popc(bi & lt)] = e[k].ref;
      if (pass && !inner) W.leafq[nleaf + __popc(bl & lt)] = ei[k];
      top += __popc(bi);
      nleaf += __popc(bl);
    }
  }
  __syncwarp();
  long long steps = 0;
  while (top > 0 || nleaf > 0) {
    if (++steps > c.max_steps) {
      overflow = true;
      return 0;
    }
    if (nleaf >= 32 || top == 0) {
      for (int q0 = 0; q0 < nleaf; q0 += 32) {
        const int nb = min(32, nleaf - q0);
        Entry le;
        le.lox = le.loy = le.loz = 1.f;
        le.hix = le.hiy = le.hiz = 0.f;  // empty
        le.minid = INT_MAX;
        le.ref = -1;
        int key = INT_MAX, src = lane;
        if (lane < nb) {
          const int ei = W.leafq[q0 + lane];
          le = load_entry(ei >= 0 ? c.nodes + ei : c.root);
          key = le.minid;
        }
        warp_sort_keys(key, src);
        for (int k = 0; k < nb; ++k) {
          const int mk = __shfl_sync(kFull, key, k);
          if (mk >= wb) break;  // warp-uniform; later leaves' IDs are larger
          const int from = __shfl_sync(kFull, src, k);
          Entry e;
          e.lox = __shfl_sync(kFull, le.lox, from);
          e.loy = __shfl_sync(kFull, le.loy, from);
          e.loz = __shfl_sync(kFull, le.loz, from);
          e.hix = __shfl_sync(kFull, le.hix, from);
          e.hiy = __shfl_sync(kFull, le.hiy, from);
          e.hiz = __shfl_sync(kFull, le.hiz, from);
          const int ref = __shfl_sync(kFull, le.ref, from);
          const bool need = act && mk < bound && nonempty(e) &&
                            lower_d2(px, py, pz, e) < r2;
          if (!__any_sync(kFull, need)) continue;
          int start, cnt;
          leaf_decode(ref, start, cnt);
          for (int j = 0; j < cnt; ++j) {
            const float4 pt = __ldg(c.pts + start + j);
            const int id = __float_as_int(pt.w);
            const bool cand = need && id < m && id < bound;
            // in an ascending leaf no later point can qualify
            if (c.sorted && !__any_sync(kFull, cand)) break;
            if (cand && exact_d2(px, py, pz, pt.x, pt.y, pt.z) < r2) {
              int pos = count < K ? count : K - 1;
              while (pos > 0 && L[pos - 1] > id) {
                L[pos] = L[pos - 1];
                --pos;
              }
              L[pos] = id;
              if (count < K) ++count;
              if (count == K) bound = L[K - 1];
            }
          }
          wb = (int)__reduce_max_sync(kFull, act ? (unsigned)bound : 0u);
        }
      }
      nleaf = 0;
      __syncwarp();
      continue;
    }
    // Pop up to 16 internal nodes; lane 2i+j tests child j of node i.
    const int P = min(top, 16);
    bool pass = false, inner = false;
    int ei = 0, ref = 0;
    if (lane < 2 * P) {
      ei = 2 * W.front[top - P + (lane >> 1)] + (lane & 1);
      const Entry e = load_entry(c.nodes + ei);
      pass = e.minid < m && e.minid < wb &&
             box_lower_d2(pk.lx, pk.ly, pk.lz, pk.hx, pk.hy, pk.hz, e) < r2;
      inner = e.ref >= 0;
      ref = e.ref;
    }
    __syncwarp();
    top -= P;
    const unsigned bi = __ballot_sync(kFull, pass && inner);
    const unsigned bl = __ballot_sync(kFull, pass && !inner);
    const int ni = __popc(bi);
    if (top + ni > FRONT) {
      overflow = true;
      return 0;
    }
    if (pass && inner) W.front[top + __popc(bi & lt)] = ref;
    if (pass && !inner) W.leafq[nleaf + __popc(bl & lt)] = ei;
    top += ni;
    nleaf += __popc(bl);
    __syncwarp();
  }
  return count;
}

template <int STACK>
__global__ void __launch_bounds__(kFWarps * 32)
    radius_frontier_kernel(QArgs a) {
  __shared__ WarpBufs<kPacketCap, 2 * STACK> wb[kFWarps];
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  Slot s = slot_setup(a, d, b);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long t0 = ((long long)blockIdx.x * kFWarps + warp) * a.pw;
  if (t0 >= s.slots) return;  // warp-uniform
  WarpBufs<kPacketCap, 2 * STACK>& W = wb[warp];
  int qi = lane < a.pw ? slot_query(s, d, (int)t0 + lane) : -1;
  bool active = qi >= 0;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (active) {
    const float* qp = a.q + 3ll * (s.qin + qi);
    px = qp[0];
    py = qp[1];
    pz = qp[2];
  }
  RadiusCtx c = radius_ctx(a, d, b, s);
  int* H = W.buf[lane];
  if (s.ovf) {  // tree-uniform: no usable tree, every query scans
    int count = 0;
    if (active) {
      atomicAdd(a.fallback, 1);
      count = scan_ordered(c, px, py, pz, H);
    }
    write_rows4(a.out, &W.buf[0][0], kPacketCap + 1, qi, count, s.qbase, c.K,
                lane);
    return;
  }
  // Queries with a non-finite coordinate have no hits (their squared
  // distances are inf or NaN) and stay out of the packet box.
  const bool live = active && finite3(px, py, pz);
  float bound = c.r2;
  int hc = 0;  // this lane's hit count (may exceed kPacketCap)
  bool overflow = false;
  const int* cut = a.f.cut + ((size_t)b * a.f.levels + s.lev) * kCutStride;
  if (__any_sync(kFull, live)) {
    Packet pk = make_packet(live, px, py, pz, bound);
    overflow = frontier_walk<false>(W, c.nodes, c.root, cut, c.pts,
                                    c.max_steps, c.m, pk, live, px, py, pz,
                                    bound, hc);
  }
  __syncwarp();
  int count = 0;
  if (!overflow) {
    bool spill = active && hc > kPacketCap;
    // ascending IDs: a sorting network in registers (no data-dependent
    // branches), sized by the warp's largest hit count
    const bool sorted_here = active && !spill;
    const int most = (int)__reduce_max_sync(kFull, sorted_here ? hc : 0);
    if (sorted_here) {
      if (most > 24)
        sort_hits<32, 32>(H, hc);
      else if (most > 20)
        sort_hits<32, 24>(H, hc);
      else if (most > 16)
        sort_hits<32, 20>(H, hc);
      else
        sort_hits<16, 16>(H, hc);
    }
    if (sorted_here) count = min(hc, c.K);
    if (__any_sync(kFull, spill)) {
      // The buffer holds kPacketCap >= K hits, so the first K IDs are all at
      // most its largest ID: the walk starts with that bound.
      int b0 = INT_MAX;
      if (spill) {
        b0 = H[0];
        for (int i = 1; i < kPacketCap; ++i) b0 = max(b0, H[i]);
        b0 += 1;
      }
      bool again = false;
      int c2 = 0;
      const bool dense =
          GSA_DENSE_WALK &&
          (int)__reduce_max_sync(kFull, spill ? (unsigned)hc : 0u) <=
              GSA_DENSE_MAX_HITS;
      if (dense)
        c2 = dense_walk<2 * STACK>(W, c, cut, spill, px, py, pz, b0, again);
      if (again || !dense) {
        again = false;
        c2 = walk_ordered<STACK>(c, spill, px, py, pz, H, W.front, again, b0);
      }
      if (spill) count = c2;
      if (again && spill) {
        atomicAdd(a.fallback, 1);
        count = scan_ordered(c, px, py, pz, H);
      }
    }
  } else {
    bool again = false;
    count = walk_ordered<STACK>(c, active, px, py, pz, H, W.front, again);
    if (again && active) {
      atomicAdd(a.fallback, 1);
      count = scan_ordered(c, px, py, pz, H);
    }
  }
  write_rows4(a.out, &W.buf[0][0], kPacketCap + 1, qi, count, s.qbase, c.K,
              lane);
}

template <int STACK>
__global__ void __launch_bounds__(kFWarps * 32)
    knn3_frontier_kernel(QArgs a) {
  __shared__ WarpBufs<kCandCap, 2 * STACK> wb[kFWarps];
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  Slot s = slot_setup(a, d, b);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long t0 = ((long long)blockIdx.x * kFWarps + warp) * a.pw;
  if (t0 >= s.slots) return;  // warp-uniform
  WarpBufs<kCandCap, 2 * STACK>& W = wb[warp];
  int qi = lane < a.pw ? slot_query(s, d, (int)t0 + lane) : -1;
  bool active = qi >= 0;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (active) {
    const float* qp = a.q + 3ll * (s.qin + qi);
    px = qp[0];
    py = qp[1];
    pz = qp[2];
  }
  KnnCtx c = knn_ctx(a, d, b, s);
  if (s.ovf) {  // tree-uniform: no usable tree, every query scans
    if (active) {
      atomicAdd(a.fallback, 1);
      write_top3(a, s, qi, scan_knn3(c, px, py, pz));
    }
    return;
  }
  const int m = c.m;
  const float inf = __int_as_float(0x7f800000);
  // Non-finite queries have no finite distance: their rows stay (inf, 0).
  const bool live = active && finite3(px, py, pz);
  float B = inf;
  // Queries in a given order are not the support's points: no window; they
  // take the per-query walk below, in packets made coherent by that order.
  if (live && !s.perm) {
    // window of the level's members around the query's member rank (a query
    // that is not a support point of this tree uses the first members)
    const int nl = level_size(d.n, s.lev);
    int r0 = qi < d.n ? __ldg(a.f.wrank + (size_t)(d.p0 + qi) * a.f.levels + s.lev) : 0;
    int lo = max(0, min(r0 - kWindow, nl - 2 * kWindow));
    int hi = min(nl, lo + 2 * kWindow);
    float w0 = inf, w1 = inf, w2 = inf;
    for (int k = lo; k < hi; ++k) {
      float4 pt = __ldg(c.pts + k);
      if (__float_as_int(pt.w) >= m) continue;
      float v = exact_d2(px, py, pz, pt.x, pt.y, pt.z);
      if (v < w2) {
        if (v < w1) {
          w2 = w1;
          if (v < w0) {
            w1 = w0;
            w0 = v;
          } else {
            w1 = v;
          }
        } else {
          w2 = v;
        }
      }
    }
    B = w2;  // inf unless three finite distances were seen
  }
  const bool inpk = live && B < inf;
  int nc = 0;  // this lane's candidates
  bool overflow = false;
  if (__any_sync(kFull, inpk)) {
    Packet pk = make_packet(inpk, px, py, pz, B);
    const int* cut = a.f.cut + ((size_t)b * a.f.levels + s.lev) * kCutStride;
    overflow = frontier_walk<true>(W, c.nodes, c.root, cut, c.pts, c.max_steps,
                                   m, pk, inpk, px, py, pz, B, nc);
  }
  __syncwarp();
  Top3 t = empty_top3();
  if (!overflow && inpk) t = cut_candidates(c.pts, W.buf[lane], nc, px, py, pz);
  // lanes without a finite window bound, or every lane after an overflow
  bool rest = live && (overflow || !inpk);
  if (__any_sync(kFull, rest)) {
    Top3 u = empty_top3();
    bool again = walk_knn3<STACK>(c, rest, px, py, pz, u, W.front);
    if (again && rest) {
      atomicAdd(a.fallback, 1);
      u = scan_knn3(c, px, py, pz);
    }
    if (rest) t = u;
  }
  if (active) write_top3(a, s, qi, t);
}

// ---------------------------------------------------------------------------
// Warp-cooperative original-order scans for small support prefixes.  One
// warp answers one query: the 32 lanes test 32 consecutive support IDs, a
// ballot orders the hits by ID, and the scan stops once K are found (radius)
// or after m points (3NN, per-lane top-3 merged across the warp).  A warp's
// serial work is m/32 steps instead of a tree walk, and there is one warp per
// query instead of one per 32, which suits small prefixes with few queries.
constexpr int kScanWarps = 8;

__global__ void __launch_bounds__(kScanWarps * 32)
    radius_scan_kernel(QArgs a) {
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  int qbase = a.qseg ? a.qseg[b] : 0;
  int qin = a.qstart ? a.qstart[b] : qbase;
  int Q = a.qseg ? a.qseg[b + 1] - qbase : a.nq;
  int m = a.m > 0 ? a.m : level_size(d.n, a.level);
  int lane = threadIdx.x & 31;
  long long qi = (long long)blockIdx.x * kScanWarps + (threadIdx.x >> 5);
  if (qi >= Q) return;  // warp-uniform
  const float* qp = a.q + 3ll * (qin + qi);
  float px = qp[0], py = qp[1], pz = qp[2];
  const float r2 = __fmul_rn(a.radius, a.radius);
  const int K = a.ns;
  const float* xs = a.f.x + 3ll * d.p0;
  int* row = a.out + (size_t)(qbase + qi) * K;
  int count = 0, first = 0;
  for (int base = 0; base < m && count < K; base += 32) {
    int id = base + lane;
    bool hit = false;
    if (id < m) {
      const float* p = xs + 3ll * id;
      hit = exact_d2(px, py, pz, p[0], p[1], p[2]) < r2;
    }
    unsigned bal = __ballot_sync(kFull, hit);
    if (!bal) continue;
    if (!count) first = base + __ffs(bal) - 1;
    int pos = count + __popc(bal & ((1u << lane) - 1u));
    if (hit && pos < K) row[pos] = id;
    count += __popc(bal);
  }
  count = min(count, K);
  for (int k = count + lane; k < K; k += 32) row[k] = count ? first : 0;
}

__global__ void __launch_bounds__(kScanWarps * 32)
    knn3_scan_kernel(QArgs a) {
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  int qbase = a.qseg ? a.qseg[b] : 0;
  int qin = a.qstart ? a.qstart[b] : qbase;
  int Q = a.qseg ? a.qseg[b + 1] - qbase : a.nq;
  int m = a.m > 0 ? a.m : level_size(d.n, a.level);
  int lane = threadIdx.x & 31;
  long long qi = (long long)blockIdx.x * kScanWarps + (threadIdx.x >> 5);
  if (qi >= Q) return;
  const float* qp = a.q + 3ll * (qin + qi);
  float px = qp[0], py = qp[1], pz = qp[2];
  const float inf = __int_as_float(0x7f800000);
  float d0 = inf, d1 = inf, d2 = inf;
  int i0 = INT_MAX, i1 = INT_MAX, i2 = INT_MAX;
  const float* xs = a.f.x + 3ll * d.p0;
  for (int id = lane; id < m; id += 32) {
    const float* p = xs + 3ll * id;
    insert3(exact_d2(px, py, pz, p[0], p[1], p[2]), id, d0, d1, d2, i0, i1, i2);
  }
  for (int o = 16; o; o >>= 1) {
    float e0 = __shfl_xor_sync(kFull, d0, o), e1 = __shfl_xor_sync(kFull, d1, o),
          e2 = __shfl_xor_sync(kFull, d2, o);
    int j0 = __shfl_xor_sync(kFull, i0, o), j1 = __shfl_xor_sync(kFull, i1, o),
        j2 = __shfl_xor_sync(kFull, i2, o);
    insert3(e0, j0, d0, d1, d2, i0, i1, i2);
    insert3(e1, j1, d0, d1, d2, i0, i1, i2);
    insert3(e2, j2, d0, d1, d2, i0, i1, i2);
  }
  if (lane < 3) {
    float v = lane == 0 ? d0 : (lane == 1 ? d1 : d2);
    int id = lane == 0 ? i0 : (lane == 1 ? i1 : i2);
    size_t o = (size_t)(qbase + qi) * 3 + lane;
    a.dout[o] = v;
    a.out[o] = id == INT_MAX ? 0 : id;
  }
}

// Largest support prefix any tree of the launch searches (host side).
int max_prefix(const Forest& f, const QuerySet& qs) {
  if (!qs.qseg_host) return qs.m;
  int best = 0;
  for (int b = 0; b < f.B; ++b) {
    if (qs.qseg_host[b + 1] == qs.qseg_host[b]) continue;
    best = std::max(best, qs.m ? qs.m : level_size(f.hdesc[b].n, qs.level));
  }
  return best;
}

long long max_queries(const Forest& f, const QuerySet& qs) {
  if (!qs.qseg_host) return qs.nq;
  long long best = 0;
  for (int b = 0; b < f.B; ++b)
    best = std::max<long long>(best, qs.qseg_host[b + 1] - qs.qseg_host[b]);
  return best;
}

// Slots (query positions walked by warps) of one tree, as slot_setup.
long long tree_slots(int n, int levels, int nq) {
  if (nq > n) return nq;
  int l = 0;
  while (l + 1 < levels && level_size(n, l + 1) >= nq) ++l;
  return level_size(n, l);
}

// Largest slot count over the trees, from host-side query offsets.
long long max_slots(const Forest& f, const QuerySet& qs) {
  const int* qseg_host = qs.qseg_host;
  const int nq = qs.nq;
  if (qs.morton) return nq;  // single tree, every query row once
  if (!qseg_host) return nq > 0 ? tree_slots(f.hdesc[0].n, f.levels, nq) : 0;
  long long best = 0;
  for (int b = 0; b < f.B; ++b) {
    int q = qseg_host[b + 1] - qseg_host[b];
    if (q > 0) best = std::max(best, tree_slots(f.hdesc[b].n, f.levels, q));
  }
  return best;
}

QArgs make_args(const Forest& f, const QuerySet& qs) {
  QArgs a;
  a.f = f.view();
  a.q = qs.q;
  a.qstart = qs.qstart;
  a.qseg = qs.qseg;
  a.nq = qs.nq;
  a.m = qs.m;
  a.level = qs.level;
  a.radius = 0.f;
  a.ns = 0;
  a.out = nullptr;
  a.dout = nullptr;
  a.fallback = nullptr;
  a.pw = 32;
  a.qperm = nullptr;
  return a;
}

}  // namespace

namespace {

int sm_count() {
  // per device, filled on first use; host threads may race to fill an entry
  // and all store the same value
  static std::atomic<int> cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// Queries per warp of a frontier launch.  A packet of 32 queries shares one
// walk of the tree, which is the cheapest per query; a launch whose grid
// would hold fewer than 16 warps per SM (a single scene) takes narrower
// packets (16, 8, 4, then 2 queries) so that more warps walk at once: each
// walk is shorter and the launch's latency falls, at some cost in
// instructions per query (one scene of 24,000 points: radius stage 0 108 ->
// 90 us, 3NN stage 0 57 -> 51 us; radius stage 1 at 6,000 queries 32.6 ->
// 24.6 us and stage 2 22.5 -> 18.5 us with packets down to 2; 8 or more such
// scenes keep 32).
#ifndef GSA_PACKET_MIN
#define GSA_PACKET_MIN 2
#endif
constexpr int kPacketMin = GSA_PACKET_MIN;
#ifndef GSA_PACKET_FILL_WARPS
#define GSA_PACKET_FILL_WARPS 16
#endif
constexpr int kPacketFillWarps = GSA_PACKET_FILL_WARPS;  // warps per SM below which packets narrow
// Packets (warps) of a tree launch at `pw` queries per warp.
long long launch_warps(const Forest& f, long long slots, int pw) {
  return (slots + kFWarps * pw - 1) / (kFWarps * pw) * kFWarps * f.B;
}
int packet_width(const Forest& f, long long slots) {
  int pw = 32;
  while (pw > kPacketMin &&
         launch_warps(f, slots, pw) < (long long)kPacketFillWarps * sm_count())
    pw >>= 1;
  return pw;
}

// The warp scan answers a launch when its support prefixes are small, or
// when the tree kernels' grid would not fill the SMs (few queries) and the
// scan's work, queries x prefix, stays bounded (a 1,000,000-point scene's
// 15,625 level-3 points against its 3,906-point prefix: 0.36 ms on the tree
// grid of 122 blocks).  `narrow`: count the tree grid at the launch's packet
// width (radius launches; one scene's 6,000 level-1 radius queries then take
// the tree, 30 us against 53 us for the scan), else at 32 queries per warp
// (3NN, whose scan stays faster there: 28 us against 38 us).  scan_max 0
// keeps every launch on the tree.
bool prefer_scan(const Forest& f, const QuerySet& qs, int scan_max,
                 bool narrow) {
  const int m = max_prefix(f, qs);
  if (m <= scan_max) return true;
  if (scan_max <= 0) return false;
  long long slots = max_slots(f, qs);
  const int pw = narrow ? packet_width(f, slots) : 32;
  if (launch_warps(f, slots, pw) >= 4ll * sm_count()) return false;
  long long q = qs.qseg_host ? qs.qseg_host[f.B] : qs.nq;
  return q * (long long)m <= (1ll << 26);
}

}  // namespace

cudaError_t launch_radius(const Forest& f, const QuerySet& qs, float radius,
                          int ns, int* out, int* fallback, cudaStream_t s) {
  QArgs a = make_args(f, qs);
  a.radius = radius;
  a.ns = ns;
  a.out = out;
  a.fallback = fallback;
  if (prefer_scan(f, qs, GSA_RADIUS_SCAN_MAX, true)) {
    long long nq = max_queries(f, qs);
    if (nq <= 0) return cudaSuccess;
    dim3 grid((unsigned)((nq + kScanWarps - 1) / kScanWarps), f.B);
    count_launches();
    radius_scan_kernel<<<grid, kScanWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
  }
  long long slots = max_slots(f, qs);
  if (slots <= 0) return cudaSuccess;
  void* block = nullptr;
  if (qs.morton) {
    cudaError_t e = sort_query_rows(qs.q, qs.nq, &a.qperm, &block, s);
    if (e) {
      pool_free(block, s);
      return e;
    }
  }
  count_launches();
  if (GSA_RADIUS_FRONTIER) {
    a.pw = packet_width(f, slots);
    dim3 grid((unsigned)((slots + kFWarps * a.pw - 1) / (kFWarps * a.pw)), f.B);
    radius_frontier_kernel<GSA_STACK><<<grid, kFWarps * 32, 0, s>>>(a);
  } else {
    dim3 grid((unsigned)((slots + kQThreads - 1) / kQThreads), f.B);
    radius_kernel<GSA_STACK><<<grid, kQThreads, 0, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  cudaError_t fe = pool_free(block, s);
  return e ? e : fe;
}

cudaError_t launch_knn3(const Forest& f, const QuerySet& qs, float* d, int* ix,
                        int* fallback, cudaStream_t s) {
  QArgs a = make_args(f, qs);
  a.dout = d;
  a.out = ix;
  a.fallback = fallback;
  if (prefer_scan(f, qs, GSA_KNN_SCAN_MAX, false)) {
    long long nq = max_queries(f, qs);
    if (nq <= 0) return cudaSuccess;
    dim3 grid((unsigned)((nq + kScanWarps - 1) / kScanWarps), f.B);
    count_launches();
    knn3_scan_kernel<<<grid, kScanWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
  }
  long long slots = max_slots(f, qs);
  if (slots <= 0) return cudaSuccess;
  void* block = nullptr;
  if (qs.morton) {
    cudaError_t e = sort_query_rows(qs.q, qs.nq, &a.qperm, &block, s);
    if (e) {
      pool_free(block, s);
      return e;
    }
  }
  count_launches();
  if (GSA_KNN_FRONTIER) {
    a.pw = packet_width(f, slots);
    dim3 grid((unsigned)((slots + kFWarps * a.pw - 1) / (kFWarps * a.pw)), f.B);
    knn3_frontier_kernel<GSA_STACK><<<grid, kFWarps * 32, 0, s>>>(a);
  } else {
    dim3 grid((unsigned)((slots + kQThreads - 1) / kQThreads), f.B);
    knn3_kernel<GSA_STACK><<<grid, kQThreads, 0, s>>>(a);
  }
  cudaError_t e = cudaGetLastError();
  cudaError_t fe = pool_free(block, s);
  return e ? e : fe;
}

}  // namespace gsa
