// SPDX-License-Identifier: Apache-2.0
// Exact ordered radius query and exact 3NN query over a prefix-bounds forest.
//
// Semantics follow GSA csrc/gsa_bvh.cu:282-343 (radius_ordered) and
// csrc/gsa_bvh.cu:149-211 (query3): the first `ns` qualifying support IDs
// < m in ascending ID order with d2 < r*r (pad with the first, zero row when
// none); the three smallest finite squared distances in (d2, id) order,
// missing entries (inf, 0).  Results do not depend on traversal order.
//
// Execution model (B200): one warp traverses the tree for 32 queries at once
// ("packet" traversal).  Queries are visited in the tree's leaf order (for a
// query array that is a prefix of the support, neighbouring lanes hold
// neighbouring points), so the 32 lanes need nearly the same nodes; a node is
// entered when any lane needs it, node entries and leaf points are loaded
// once per warp as 16-byte broadcast loads, and each lane tests its own query.
// The radius descent order is ascending subtree minimum ID (stored order of
// the children), which makes the "K found and minid >= K-th ID" early exit of
// the reference effective.  The warp stack lives in shared memory; a stack
// overflow (impossible for STACK >= 97 on a Karras tree of 64-bit keys) falls
// back to the exact original-order scan and is counted, as in the reference.
#include <algorithm>
#include "forest.cuh"

#ifndef GSA_STACK
#define GSA_STACK 128
#endif
// Support prefixes up to these sizes are answered by the warp scans below
// instead of a tree walk (same results; fewer serial steps per warp).
#ifndef GSA_RADIUS_SCAN_MAX
#define GSA_RADIUS_SCAN_MAX 2048
#endif
#ifndef GSA_KNN_SCAN_MAX
#define GSA_KNN_SCAN_MAX 1024
#endif
// Tree-walk radius kernel: 1 culls with the warp's packet box and processes
// leaves as dense (query, point) pairs (radius_frontier_kernel); 0 is the
// ordered per-query packet walk (radius_kernel) throughout.
#ifndef GSA_RADIUS_DENSE
#define GSA_RADIUS_DENSE 1
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
  const int* order;
};

__device__ __forceinline__ Slot slot_setup(const QArgs& a, const TreeDesc& d,
                                           int b) {
  Slot s;
  s.qbase = a.qseg ? a.qseg[b] : 0;
  s.qin = a.qstart ? a.qstart[b] : s.qbase;
  s.Q = a.qseg ? a.qseg[b + 1] - s.qbase : a.nq;
  s.m = a.m > 0 ? a.m : level_size(d.n, a.level);
  s.lev = a.level < 0 ? 0 : a.level;
  int ql = s.Q <= d.n ? query_level(d.n, a.f.levels, s.Q) : 0;
  s.slots = s.Q <= d.n ? level_size(d.n, ql) : s.Q;
  s.order = a.f.qorder + d.q0 + level_offset(d.n, ql);
  return s;
}

__device__ __forceinline__ int slot_query(const Slot& s, const TreeDesc& d,
                                          int t) {
  if (t >= s.slots) return -1;
  int qi = t < d.n ? __ldg(s.order + t) : t;
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
// Returns the lane's count; sets overflow (warp-uniform) on stack overflow.
template <int STACK>
__device__ int walk_ordered(const RadiusCtx& c, bool active, float px,
                            float py, float pz, int* L, int* stk,
                            bool& overflow) {
  const int K = c.K, m = c.m;
  const float r2 = c.r2;
  int count = 0, bound = INT_MAX;
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

__device__ __forceinline__ RadiusCtx radius_ctx(const QArgs& a,
                                                const TreeDesc& d, int b,
                                                const Slot& s) {
  RadiusCtx c;
  c.nodes = a.f.nodes + d.node0 + (size_t)s.lev * (d.n - 1) * 2;
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
  bool overflow = false;
  int count = walk_ordered<STACK>(c, active, px, py, pz, L, stack[warp], overflow);
  if (overflow && active) {
    atomicAdd(a.fallback, 1);
    count = scan_ordered(c, px, py, pz, L);
  }
  write_rows(a.out, &lists[warp][0][0], 33, qi, count, s.qbase, c.K, lane);
}

// Packet-frontier variant.  A warp's 32 queries are neighbours in leaf order,
// so the tree is culled once for all of them against the box of the warp's
// finite queries (box_lower_d2), 32 child entries per step (one per lane)
// from a warp frontier stack, instead of a per-query test of two children
// per step.  Leaves that survive are queued; each queued leaf is then tested
// per query against its own box and processed as (query x point) pairs with
// the leaf's points held one per lane (w = leaf count rounded up to a power
// of two, 32/w queries per step).  Hits go unordered into per-query shared
// buffers, ranked by ballot, and are sorted at the end.  A frontier that
// would exceed its stack, or a query with more than kPacketCap hits, is
// answered by the ordered walk.  Results are identical to radius_kernel.
constexpr int kFWarps = 4;
constexpr int kPacketCap = 32;  // per-query hit buffer; holds a K-list (K<=32)

template <int STACK>
__global__ void __launch_bounds__(kFWarps * 32)
    radius_frontier_kernel(QArgs a) {
  constexpr int kFront = 2 * STACK;
  __shared__ int hits[kFWarps][32][kPacketCap + 1];
  __shared__ float4 qbuf[kFWarps][32];
  __shared__ int amap[kFWarps][32];
  __shared__ int leafq[kFWarps][64];
  __shared__ int front[kFWarps][kFront];
  int b = blockIdx.y;
  TreeDesc d = a.f.desc[b];
  Slot s = slot_setup(a, d, b);
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long t0 = ((long long)blockIdx.x * kFWarps + warp) * 32;
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
  const int m = c.m;
  const float r2 = c.r2;
  const unsigned lt = (1u << lane) - 1u;
  int* H = hits[warp][lane];
  int* stk = front[warp];
  int* lq = leafq[warp];
  // Queries with a non-finite coordinate have no hits (their squared
  // distances are inf or NaN) and stay out of the packet box.
  const bool live = active && finite3(px, py, pz);
  qbuf[warp][lane] = make_float4(px, py, pz, 0.f);
  int hc = 0;  // this lane's hit count (may exceed kPacketCap)
  bool overflow = false;
  if (__any_sync(kFull, live)) {
    const float blx = key_float(__reduce_min_sync(kFull, live ? float_key(px) : ~0u));
    const float bly = key_float(__reduce_min_sync(kFull, live ? float_key(py) : ~0u));
    const float blz = key_float(__reduce_min_sync(kFull, live ? float_key(pz) : ~0u));
    const float bhx = key_float(__reduce_max_sync(kFull, live ? float_key(px) : 0u));
    const float bhy = key_float(__reduce_max_sync(kFull, live ? float_key(py) : 0u));
    const float bhz = key_float(__reduce_max_sync(kFull, live ? float_key(pz) : 0u));
    int top = 0, nleaf = 0;
    {
      Entry root = load_entry(c.root);
      if (root.minid < m &&
          box_lower_d2(blx, bly, blz, bhx, bhy, bhz, root) < r2) {
        if (root.ref >= 0) {
          if (lane == 0) stk[0] = root.ref;
          top = 1;
        } else {
          if (lane == 0) lq[0] = -1;  // the root itself is the only leaf
          nleaf = 1;
        }
      }
    }
    __syncwarp();
    long long steps = 0;
    while (top > 0 || nleaf > 0) {
      if (++steps > c.max_steps) {
        overflow = true;
        break;
      }
      if (top > 0) {
        // Pop up to 16 internal nodes; lane 2i+j tests child j of node i.
        int P = min(top, 16);
        bool pass = false, inner = false;
        int ei = 0, ref = 0;
        if (lane < 2 * P) {
          ei = 2 * stk[top - P + (lane >> 1)] + (lane & 1);
          Entry e = load_entry(c.nodes + ei);
          pass = e.minid < m &&
                 box_lower_d2(blx, bly, blz, bhx, bhy, bhz, e) < r2;
          inner = e.ref >= 0;
          ref = e.ref;
        }
        __syncwarp();
        top -= P;
        unsigned bi = __ballot_sync(kFull, pass && inner);
        unsigned bl = __ballot_sync(kFull, pass && !inner);
        int ni = __popc(bi);
        if (top + ni > kFront) {
          overflow = true;
          break;
        }
        if (pass && inner) stk[top + __popc(bi & lt)] = ref;
        if (pass && !inner) lq[nleaf + __popc(bl & lt)] = ei;
        top += ni;
        nleaf += __popc(bl);
        __syncwarp();
      }
      if (nleaf < 32 && top > 0) continue;
      for (int li = 0; li < nleaf; ++li) {
        int ei = lq[li];
        Entry e = load_entry(ei >= 0 ? c.nodes + ei : c.root);
        bool need = live && lower_d2(px, py, pz, e) < r2;
        unsigned M = __ballot_sync(kFull, need);
        if (!M) continue;
        int start, cnt;
        leaf_decode(e.ref, start, cnt);
        const int nA = __popc(M);
        const int mine = __popc(M & lt);
        if (need) amap[warp][mine] = lane;
        __syncwarp();
        const int logw = cnt <= 1 ? 0 : 32 - __clz(cnt - 1);
        const int w = 1 << logw, per = 32 >> logw;
        const int k = lane >> logw, j = lane & (w - 1);
        const unsigned seg0 = w == 32 ? kFull : (1u << w) - 1u;
        float4 pt = make_float4(0.f, 0.f, 0.f, __int_as_float(INT_MAX));
        if (j < cnt) pt = __ldg(c.pts + start + j);
        const int id = __float_as_int(pt.w);
        const bool pv = j < cnt && id < m;
        for (int base = 0; base < nA; base += per) {
          int idx = base + k;
          bool valid = pv && idx < nA;
          int q = amap[warp][idx < nA ? idx : 0];
          float4 qc = qbuf[warp][q];
          bool hit = valid && exact_d2(qc.x, qc.y, qc.z, pt.x, pt.y, pt.z) < r2;
          unsigned hm = __ballot_sync(kFull, hit);
          if (!hm) continue;  // warp-uniform
          int at = __shfl_sync(kFull, hc, q);
          int slot = at + __popc(hm & (seg0 << (k << logw)) & lt);
          if (hit && slot < kPacketCap) hits[warp][q][slot] = id;
          int mk = mine - base;
          if (need && mk >= 0 && mk < per)
            hc += __popc(hm & (seg0 << (mk << logw)));
        }
        __syncwarp();
      }
      nleaf = 0;
    }
  }
  __syncwarp();
  int count = 0;
  if (!overflow) {
    bool spill = active && hc > kPacketCap;
    if (active && !spill) {
      for (int i = 1; i < hc; ++i) {  // ascending IDs
        int v = H[i], pos = i;
        while (pos > 0 && H[pos - 1] > v) {
          H[pos] = H[pos - 1];
          --pos;
        }
        H[pos] = v;
      }
      count = min(hc, c.K);
    }
    if (__any_sync(kFull, spill)) {
      bool again = false;
      int c2 = walk_ordered<STACK>(c, spill, px, py, pz, H, stk, again);
      if (spill) count = c2;
      if (again && spill) {
        atomicAdd(a.fallback, 1);
        count = scan_ordered(c, px, py, pz, H);
      }
    }
  } else {
    bool again = false;
    count = walk_ordered<STACK>(c, active, px, py, pz, H, stk, again);
    if (again && active) {
      atomicAdd(a.fallback, 1);
      count = scan_ordered(c, px, py, pz, H);
    }
  }
  write_rows(a.out, &hits[warp][0][0], kPacketCap + 1, qi, count, s.qbase,
             c.K, lane);
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
  const int m = s.m;
  const float inf = __int_as_float(0x7f800000);
  float d0 = inf, d1 = inf, d2 = inf;
  int i0 = INT_MAX, i1 = INT_MAX, i2 = INT_MAX;
  int* stk = stack[warp];
  const Entry* nodes = a.f.nodes + d.node0 + (size_t)s.lev * (d.n - 1) * 2;
  const float4* pts = level_pts(a.f, d, s.lev);
  const bool sorted = s.lev == 0;  // leaf IDs ascend
  Entry cur = load_entry(a.f.root + b * a.f.levels + s.lev);
  bool need = active && cur.minid < m && nonempty(cur) &&
              lower_d2(px, py, pz, cur) <= d2;
  int top = 0;
  bool overflow = false;
  long long steps = 0, max_steps = 4ll * d.n + 64;
  while (true) {
    if (++steps > max_steps) {
      overflow = true;
      break;
    }
    if (!__any_sync(kFull, need)) {
      if (top == 0) break;
      int ei = stk[--top];
      cur = load_entry(nodes + ei);
      need = active && cur.minid < m && nonempty(cur) &&
             lower_d2(px, py, pz, cur) <= d2;
      continue;
    }
    if (cur.ref >= 0) {
      const Entry* ch = nodes + (size_t)cur.ref * 2;
      Entry c0 = load_entry(ch), c1 = load_entry(ch + 1);
      float l0 = lower_d2(px, py, pz, c0), l1 = lower_d2(px, py, pz, c1);
      bool n0 = need && c0.minid < m && nonempty(c0) && l0 <= d2;
      bool n1 = need && c1.minid < m && nonempty(c1) && l1 <= d2;
      unsigned b0 = __ballot_sync(kFull, n0), b1 = __ballot_sync(kFull, n1);
      if (b0 && b1) {
        unsigned both = b0 & b1;
        unsigned pref1 = __ballot_sync(kFull, n0 && n1 && l1 < l0);
        bool first1 = 2 * __popc(pref1) > __popc(both);
        if (top == STACK) {
          overflow = true;
          break;
        }
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
        float4 pt = __ldg(pts + start + j);
        int id = __float_as_int(pt.w);
        if (id >= m) {
          if (sorted) break;
          continue;
        }
        if (need)
          insert3(exact_d2(px, py, pz, pt.x, pt.y, pt.z), id, d0, d1, d2, i0,
                  i1, i2);
      }
      need = false;
    }
  }
  if (overflow && active) {
    atomicAdd(a.fallback, 1);
    d0 = d1 = d2 = inf;
    i0 = i1 = i2 = INT_MAX;
    const float* xs = a.f.x + 3ll * d.p0;
    for (int id = 0; id < m; ++id) {
      const float* p = xs + 3ll * id;
      insert3(exact_d2(px, py, pz, p[0], p[1], p[2]), id, d0, d1, d2, i0, i1,
              i2);
    }
  }
  if (active) {
    size_t o = (size_t)(s.qbase + qi) * 3;
    a.dout[o] = d0;
    a.dout[o + 1] = d1;
    a.dout[o + 2] = d2;
    a.out[o] = i0 == INT_MAX ? 0 : i0;
    a.out[o + 1] = i1 == INT_MAX ? 0 : i1;
    a.out[o + 2] = i2 == INT_MAX ? 0 : i2;
  }
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
long long max_slots(const Forest& f, const int* qseg_host, int nq) {
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
  return a;
}

}  // namespace

cudaError_t launch_radius(const Forest& f, const QuerySet& qs, float radius,
                          int ns, int* out, int* fallback, cudaStream_t s) {
  QArgs a = make_args(f, qs);
  a.radius = radius;
  a.ns = ns;
  a.out = out;
  a.fallback = fallback;
  if (max_prefix(f, qs) <= GSA_RADIUS_SCAN_MAX) {
    long long nq = max_queries(f, qs);
    if (nq <= 0) return cudaSuccess;
    dim3 grid((unsigned)((nq + kScanWarps - 1) / kScanWarps), f.B);
    count_launches();
    radius_scan_kernel<<<grid, kScanWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
  }
  long long slots = max_slots(f, qs.qseg_host, qs.nq);
  if (slots <= 0) return cudaSuccess;
  count_launches();
  if (GSA_RADIUS_DENSE) {
    dim3 grid((unsigned)((slots + kFWarps * 32 - 1) / (kFWarps * 32)), f.B);
    radius_frontier_kernel<GSA_STACK><<<grid, kFWarps * 32, 0, s>>>(a);
  } else {
    dim3 grid((unsigned)((slots + kQThreads - 1) / kQThreads), f.B);
    radius_kernel<GSA_STACK><<<grid, kQThreads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_knn3(const Forest& f, const QuerySet& qs, float* d, int* ix,
                        int* fallback, cudaStream_t s) {
  QArgs a = make_args(f, qs);
  a.dout = d;
  a.out = ix;
  a.fallback = fallback;
  if (max_prefix(f, qs) <= GSA_KNN_SCAN_MAX) {
    long long nq = max_queries(f, qs);
    if (nq <= 0) return cudaSuccess;
    dim3 grid((unsigned)((nq + kScanWarps - 1) / kScanWarps), f.B);
    count_launches();
    knn3_scan_kernel<<<grid, kScanWarps * 32, 0, s>>>(a);
    return cudaGetLastError();
  }
  long long slots = max_slots(f, qs.qseg_host, qs.nq);
  if (slots <= 0) return cudaSuccess;
  dim3 grid((unsigned)((slots + kQThreads - 1) / kQThreads), f.B);
  count_launches();
  knn3_kernel<GSA_STACK><<<grid, kQThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace gsa
