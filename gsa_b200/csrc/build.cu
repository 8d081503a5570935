// SPDX-License-Identifier: Apache-2.0
// Morton/LBVH forest builder with four prefix levels on one topology.
//
// Replaces the cuBQL spatial-median build + refit + prefix refit of GSA
// (csrc/gsa_bvh.cu:217-248, 60-120).  Query results never depend on the tree
// topology (ordered first-K radius and (d2, id) 3NN with conservative bounds),
// so any valid hierarchy gives bit-identical answers; this one is built with
// no host synchronisation:
//   1. per-tree bounds of the finite points          (bounds_kernel)
//   2. Morton keys (30-63 bits by tree size), local point indices (morton_kernel)
//   3. stable LSD radix sort, 8-bit passes over the key width, per tree
//      (sort_upsweep / seg_scan / sort_scatter; all trees in one launch)
//   4. Karras radix-tree topology on (key, index)    (karras_kernel)
//   5. per prefix level, the member count (IDs < n/4^l) before every sorted
//      position                            (member_count / member_prefix)
//   6. leaves = maximal subtrees of <= `leaf` points (karras_kernel emits
//      leaf records and seeds the arrival counters); per leaf, a half-warp
//      writes its points to `pts` in leaf order and ascending ID inside the
//      leaf, per level the members' IDs to the level's query order (IDs < n/4^l
//      in leaf order, a spatially coherent order for prefix queries) and
//      their points to the level's member array, and the leaf's entries
//                                                  (leaf_kernel)
//   7. bottom-up refit of the per-level child entries (box of the finite
//      members with ID < n/4^l, the subtree's minimum ID, child/leaf
//      reference; children in ascending minimum-ID order); on levels >= 1
//      every subtree with <= `leaf` members is a leaf over the level's member
//      array, so coarse levels keep full leaves      (climb_kernel: one
//      thread per climb from each node with two leaves)
#include <cooperative_groups.h>
#include <algorithm>
#include <atomic>
#include <new>
#include "forest.cuh"
#include "pool.cuh"

namespace cg = cooperative_groups;

// Trees of up to 32,768 points are keyed and sorted by one cluster launch
// (cluster_sort_kernel); 0 keeps every tree on the multi-launch path.
#ifndef GSA_CLUSTER_SORT
#define GSA_CLUSTER_SORT 1
#endif

// 1: launches with few trees sort with 2,048-position tiles (clusters of up
// to 16 CTAs); 0: always 4,096.
#ifndef GSA_SMALL_SORT_TILES
#define GSA_SMALL_SORT_TILES 1
#endif

namespace gsa {
namespace {

constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;  // 2048 keys per block
constexpr int kScanThreads = 1024;

struct DescChunk {
  TreeDesc d[256];
  int first, count;
};

__global__ void upload_desc(TreeDesc* dst, DescChunk c, unsigned* bounds) {
  int i = threadIdx.x;
  if (i < c.count) {
    dst[c.first + i] = c.d[i];
    if (bounds) {
      unsigned* b = bounds + 6 * (c.first + i);
      b[0] = b[1] = b[2] = 0xffffffffu;  // min keys
      b[3] = b[4] = b[5] = 0u;           // max keys
    }
  }
}

// Bounds over points whose three coordinates are finite (non-finite points
// can never qualify: their squared distance is inf or NaN).
constexpr int kUnroll = 4;  // points per thread and step (bounds, Morton)

__global__ void bounds_kernel(const TreeDesc* desc, const float* x,
                              unsigned* bounds) {
  TreeDesc d = desc[blockIdx.y];
  float lo[3] = {INFINITY, INFINITY, INFINITY};
  float hi[3] = {-INFINITY, -INFINITY, -INFINITY};
  const int stride = gridDim.x * blockDim.x;
  // kUnroll points per thread and step, all loaded before any is used
  for (int i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < d.n;
       i0 += kUnroll * stride) {
    float v[kUnroll][3];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * stride;
      v[u][0] = v[u][1] = v[u][2] = NAN;
      if (i < d.n) {
        const float* p = x + 3ll * (d.p0 + i);
        v[u][0] = p[0];
        v[u][1] = p[1];
        v[u][2] = p[2];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (finite3(v[u][0], v[u][1], v[u][2])) {
        for (int k = 0; k < 3; ++k) {
          lo[k] = fminf(lo[k], v[u][k]);
          hi[k] = fmaxf(hi[k], v[u][k]);
        }
      }
    }
  }
  for (int k = 0; k < 3; ++k) {
    for (int o = 16; o; o >>= 1) {
      lo[k] = fminf(lo[k], __shfl_xor_sync(kFull, lo[k], o));
      hi[k] = fmaxf(hi[k], __shfl_xor_sync(kFull, hi[k], o));
    }
  }
  if ((threadIdx.x & 31) == 0 && lo[0] <= hi[0]) {
    unsigned* b = bounds + 6 * blockIdx.y;
    for (int k = 0; k < 3; ++k) {
      atomicMin(b + k, float_key(lo[k]));
      atomicMax(b + 3 + k, float_key(hi[k]));
    }
  }
}

__device__ __forceinline__ uint64_t spread3(unsigned v) {
  uint64_t x = v & 0x1fffffu;
  x = (x | x << 32) & 0x1f00000000ffffull;
  x = (x | x << 16) & 0x1f0000ff0000ffull;
  x = (x | x << 8) & 0x100f00f00f00f00full;
  x = (x | x << 4) & 0x10c30c30c30c30c3ull;
  x = (x | x << 2) & 0x1249249249249249ull;
  return x;
}

// Morton keys use `bits` per axis, chosen from the largest tree: five more
// than a uniform distribution needs to separate its points (ceil(log2 n / 3)),
// 10..21.  The tree only has to be a valid hierarchy (equal keys are ordered
// by index), so the width only trades sort passes against tightness: 24,000
// points take 30-bit keys and four 8-bit radix passes, 1,000,000 take 36-bit
// keys and five.
int morton_bits(int max_n) {
  int lg = 0;
  while ((1ll << lg) < (long long)max_n) ++lg;
  return std::min(21, std::max(10, (lg + 2) / 3 + 5));
}

__device__ __forceinline__ unsigned quantize(float v, float lo, float scale,
                                             unsigned top) {
  float t = (v - lo) * scale;
  if (!(t >= 0.f)) return 0u;  // also NaN
  if (t >= (float)top) return top;
  return (unsigned)t;
}

__global__ void morton_kernel(const TreeDesc* desc, const float* x,
                              const unsigned* bounds, int bits,
                              uint64_t* keys, int* vals) {
  TreeDesc d = desc[blockIdx.y];
  const unsigned* b = bounds + 6 * blockIdx.y;
  const unsigned top = (1u << bits) - 1u;
  float lo[3], ext = 0.f;
  bool any = b[0] != 0xffffffffu;
  for (int k = 0; k < 3; ++k) {
    lo[k] = any ? key_float(b[k]) : 0.f;
    float h = any ? key_float(b[3 + k]) : 0.f;
    ext = fmaxf(ext, h - lo[k]);
  }
  float scale = (ext > 0.f && isfinite(ext)) ? (float)top / ext : 0.f;
  const int stride = gridDim.x * blockDim.x;
  for (int i0 = blockIdx.x * blockDim.x + threadIdx.x; i0 < d.n;
       i0 += kUnroll * stride) {
    float v[kUnroll][3];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * stride;
      if (i < d.n) {
        const float* p = x + 3ll * (d.p0 + i);
        v[u][0] = p[0];
        v[u][1] = p[1];
        v[u][2] = p[2];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int i = i0 + u * stride;
      if (i < d.n) {
        keys[d.p0 + i] = (spread3(quantize(v[u][0], lo[0], scale, top)) << 2) |
                         (spread3(quantize(v[u][1], lo[1], scale, top)) << 1) |
                         spread3(quantize(v[u][2], lo[2], scale, top));
        vals[d.p0 + i] = i;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Stable per-tree LSD radix sort of (64-bit key, int value) pairs.
// Histogram layout per tree: hist[(tree*D + digit)*max_tiles + tile].
__global__ void __launch_bounds__(kSortThreads)
    sort_upsweep(const TreeDesc* desc, const uint64_t* keys, int shift,
                 int* hist, int max_tiles) {
  __shared__ int h[256];
  TreeDesc d = desc[blockIdx.y];
  int tile = blockIdx.x;
  int base = tile * kSortTile;
  if (base >= d.n) return;
  h[threadIdx.x] = 0;
  __syncthreads();
  const uint64_t* k = keys + d.p0;
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    int idx = base + j * kSortThreads + threadIdx.x;
    if (idx < d.n) atomicAdd(&h[(k[idx] >> shift) & 255], 1);
  }
  __syncthreads();
  hist[((size_t)blockIdx.y * 256 + threadIdx.x) * max_tiles + tile] =
      h[threadIdx.x];
}

// Exclusive scan, per tree, of `digits` x tiles(tree) counters in digit-major
// order (one block per tree).  tiles(tree) = ceil(n / tile_size).
__global__ void __launch_bounds__(kScanThreads)
    seg_scan(const TreeDesc* desc, int* hist, int digits, int max_tiles,
             int tile_size) {
  __shared__ int warp_sums[32];
  int b = blockIdx.x;
  int n = desc[b].n;
  int tiles = (n + tile_size - 1) / tile_size;
  int total = digits * tiles;
  int per = (total + kScanThreads - 1) / kScanThreads;
  int start = threadIdx.x * per;
  int end = min(start + per, total);
  int* base = hist + (size_t)b * digits * max_tiles;
  auto at = [&](int e) -> int& {
    return base[(size_t)(e / tiles) * max_tiles + (e % tiles)];
  };
  int sum = 0;
  for (int e = start; e < end; ++e) sum += at(e);
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = sum;
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = warp_sums[lane];
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(kFull, v, o);
      if (lane >= o) v += u;
    }
    warp_sums[lane] = v;  // inclusive
  }
  __syncthreads();
  int run = incl - sum + (warp ? warp_sums[warp - 1] : 0);
  for (int e = start; e < end; ++e) {
    int c = at(e);
    at(e) = run;
    run += c;
  }
}

__global__ void __launch_bounds__(kSortThreads)
    sort_scatter(const TreeDesc* desc, const uint64_t* kin, const int* vin,
                 uint64_t* kout, int* vout, const int* hist, int shift,
                 int max_tiles) {
  __shared__ int cnt[256];
  __shared__ int goff[256];
  __shared__ int wcnt[kSortThreads / 32][256];
  TreeDesc d = desc[blockIdx.y];
  int tile = blockIdx.x;
  int base = tile * kSortTile;
  if (base >= d.n) return;
  int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  cnt[tid] = 0;
  goff[tid] = hist[((size_t)blockIdx.y * 256 + tid) * max_tiles + tile];
#pragma unroll
  for (int w = 0; w < kSortThreads / 32; ++w) wcnt[w][tid] = 0;
  __syncthreads();
  const uint64_t* k = kin + d.p0;
  const int* v = vin + d.p0;
  uint64_t* ko = kout + d.p0;
  int* vo = vout + d.p0;
  // the tile's keys and values in one round trip, then ranked 256 at a time
  uint64_t keys[kSortItems];
  int vals[kSortItems];
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    int idx = base + j * kSortThreads + tid;
    keys[j] = idx < d.n ? k[idx] : 0;
    vals[j] = idx < d.n ? v[idx] : 0;
  }
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    int idx = base + j * kSortThreads + tid;
    bool valid = idx < d.n;
    uint64_t key = keys[j];
    int val = vals[j];
    int digit = valid ? (int)((key >> shift) & 255) : 256 + lane;
    unsigned peers = __match_any_sync(kFull, digit);
    int lower = __popc(peers & ((1u << lane) - 1u));
    if (valid && lower == 0) wcnt[warp][digit] = __popc(peers);
    __syncthreads();
    if (valid) {
      int r = goff[digit] + cnt[digit] + lower;
      for (int w = 0; w < warp; ++w) r += wcnt[w][digit];
      ko[r] = key;
      vo[r] = val;
    }
    __syncthreads();
    int s = 0;
#pragma unroll
    for (int w = 0; w < kSortThreads / 32; ++w) {
      s += wcnt[w][tid];
      wcnt[w][tid] = 0;
    }
    cnt[tid] += s;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Trees of up to kClusterMaxPoints points: bounds, Morton keys, the four
// radix passes and the per-level member offsets in ONE launch.  A thread-block
// cluster owns one tree, each CTA a tile of kCTile consecutive positions; the
// CTAs exchange bounds, digit histograms and member counts through
// distributed shared memory and scatter keys straight into the destination
// CTA's buffer, with cluster barriers between the steps.  Inside a tile each
// warp owns kCItems * 32 consecutive positions, so a warp ranks its items
// against its own running digit counts (peers found by eight ballots over
// the digit bits, no block barrier per item row) and one scan over the warps
// per digit places them; reads of the other CTAs' bounds, histograms and
// member counts are issued together, one remote round trip each.  The
// multi-launch path (bounds_kernel ... member_prefix, 14 launches) does the
// same work for larger trees.  Keys are at most 30 bits here (morton_bits of
// n <= 32768 is 10), so they live in shared memory as 32-bit words; the output
// (64-bit keys, local indices, member offsets) equals the multi-launch path's.
constexpr int kCThreads = 512;
constexpr int kClusterMaxPoints = 32768;     // 8 tiles of 4096 or 16 of 2048
constexpr int kCWarps = kCThreads / 32;

// ITEMS positions per thread: tiles of 512 * ITEMS positions, at most
// kClusterMaxPoints / tile CTAs per cluster (8, the portable size, at
// ITEMS = 8; 16 at ITEMS = 4, for launches with few trees).
template <int ITEMS>
struct ClusterSmem {
  static constexpr int kCTile = kCThreads * ITEMS;
  unsigned keys[kCTile];   // the tile's keys in position order (scatter target)
  int vals[kCTile];
  int wcnt[kCWarps][256];  // per-warp digit counts, then their exclusive scan
  int hist[256];           // this tile's digit counts (read by the cluster)
  int goff[256];
  unsigned bnd[6];         // this tile's bounds keys (read by the cluster)
  unsigned gbnd[6];        // the tree's bounds keys
  int lcnt[kMaxLevels];    // this tile's member counts (read by the cluster)
  int wsum[kCWarps];
  int wmem[kCWarps][kMaxLevels];  // members per warp, then their exclusive scan
};

// Position of item j of a lane inside its CTA's tile (warp-major).
template <int ITEMS>
__device__ __forceinline__ int cpos(int warp, int j, int lane) {
  return warp * (ITEMS * 32) + j * 32 + lane;
}

// MINB: resident CTAs per SM the register budget is cut for (2: 64
// registers; 3: 40, with spills, so that the 384 tiles of 64 rooms run as
// one wave of three CTAs per SM instead of two waves of two).
template <int ITEMS, int MINB>
__global__ void __launch_bounds__(kCThreads, MINB)
    cluster_sort_kernel(const TreeDesc* desc, const float* x, int bits,
                        int levels, uint64_t* keys_out, int* vals_out,
                        int* pref, int N) {
  constexpr int kCItems = ITEMS;
  constexpr int kCTile = kCThreads * ITEMS;
  constexpr int kClusterMax = kClusterMaxPoints / kCTile;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using Smem = ClusterSmem<ITEMS>;
  Smem& S = *reinterpret_cast<Smem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int cs = (int)cluster.num_blocks();
  const TreeDesc d = desc[blockIdx.y];
  const int n = d.n;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned lt = (1u << lane) - 1u;
  const int base = rank * kCTile;

  // 1. bounds of the finite points (order-preserving keys, as bounds_kernel)
  float px[kCItems], py[kCItems], pz[kCItems];
  unsigned lo[3] = {~0u, ~0u, ~0u}, hi[3] = {0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < kCItems; ++j) {
    const int i = base + cpos<ITEMS>(warp, j, lane);
    px[j] = py[j] = pz[j] = NAN;
    if (i < n) {
      const float* q = x + 3ll * (d.p0 + i);
      px[j] = q[0];
      py[j] = q[1];
      pz[j] = q[2];
    }
    if (finite3(px[j], py[j], pz[j])) {
      lo[0] = min(lo[0], float_key(px[j]));
      lo[1] = min(lo[1], float_key(py[j]));
      lo[2] = min(lo[2], float_key(pz[j]));
      hi[0] = max(hi[0], float_key(px[j]));
      hi[1] = max(hi[1], float_key(py[j]));
      hi[2] = max(hi[2], float_key(pz[j]));
    }
  }
  if (tid < 6) S.bnd[tid] = tid < 3 ? ~0u : 0u;
  __syncthreads();
  for (int k = 0; k < 3; ++k) {
    lo[k] = __reduce_min_sync(kFull, lo[k]);
    hi[k] = __reduce_max_sync(kFull, hi[k]);
  }
  if (lane == 0) {
    for (int k = 0; k < 3; ++k) {
      atomicMin(&S.bnd[k], lo[k]);
      atomicMax(&S.bnd[3 + k], hi[k]);
    }
  }
  cluster.sync();
  // thread k < 6 reads bound k of every CTA of the cluster (all loads in
  // flight at once) and leaves the cluster-wide value in gbnd
  if (tid < 6) {
    unsigned v[kClusterMax];
#pragma unroll
    for (int c = 0; c < kClusterMax; ++c)
      v[c] = c < cs ? cluster.map_shared_rank(S.bnd, c)[tid] : S.bnd[tid];
    unsigned r = v[0];
#pragma unroll
    for (int c = 1; c < kClusterMax; ++c) r = tid < 3 ? min(r, v[c]) : max(r, v[c]);
    S.gbnd[tid] = r;
  }
  __syncthreads();
  unsigned bk[6];
#pragma unroll
  for (int k = 0; k < 6; ++k) bk[k] = S.gbnd[k];

  // 2. Morton keys (as morton_kernel) and local indices, in registers
  unsigned key[kCItems];
  int val[kCItems];
  {
    const unsigned top = (1u << bits) - 1u;
    const bool any = bk[0] != 0xffffffffu;
    float l3[3], ext = 0.f;
    for (int k = 0; k < 3; ++k) {
      l3[k] = any ? key_float(bk[k]) : 0.f;
      const float h = any ? key_float(bk[3 + k]) : 0.f;
      ext = fmaxf(ext, h - l3[k]);
    }
    const float scale = (ext > 0.f && isfinite(ext)) ? (float)top / ext : 0.f;
#pragma unroll
    for (int j = 0; j < kCItems; ++j) {
      key[j] = (unsigned)((spread3(quantize(px[j], l3[0], scale, top)) << 2) |
                          (spread3(quantize(py[j], l3[1], scale, top)) << 1) |
                          spread3(quantize(pz[j], l3[2], scale, top)));
      val[j] = base + cpos<ITEMS>(warp, j, lane);
    }
  }

  // 3. stable LSD radix passes over 8-bit digits.  Item j of a lane sits at
  // tile position cpos<ITEMS>(warp, j, lane) at the start of every pass.
  const int passes = (3 * bits + 7) / 8;
  for (int pass = 0; pass < passes; ++pass) {
    const int shift = 8 * pass;
    int* wc = S.wcnt[warp];
    for (int e = lane; e < 256; e += 32) wc[e] = 0;
    __syncwarp();
    int rk[kCItems];
#pragma unroll
    for (int j = 0; j < kCItems; ++j) {
      const bool valid = base + cpos<ITEMS>(warp, j, lane) < n;
      const int digit = valid ? (int)((key[j] >> shift) & 255) : 256 + lane;
      // lanes with this lane's digit: eight ballots over the digit bits
      unsigned peers = __ballot_sync(kFull, valid);
#pragma unroll
      for (int bit = 0; bit < 8; ++bit) {
        const unsigned bb = __ballot_sync(kFull, (digit >> bit) & 1);
        peers &= ((digit >> bit) & 1) ? bb : ~bb;
      }
      if (!valid) peers = 1u << lane;
      const int lower = __popc(peers & lt);
      rk[j] = valid ? wc[digit] + lower : 0;
      __syncwarp();
      if (valid && lower == 0) wc[digit] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    if (tid < 256) {  // tile histogram; per digit, warps' exclusive offsets
      int run = 0;
      for (int w = 0; w < kCWarps; ++w) {
        const int c = S.wcnt[w][tid];
        S.wcnt[w][tid] = run;
        run += c;
      }
      S.hist[tid] = run;
    }
    cluster.sync();  // every tile's histogram complete, every buffer read
    if (tid < 256) {
      // digits below tid over the whole tree, plus digit tid in lower tiles
      int below = 0, total = 0, v[kClusterMax];
#pragma unroll
      for (int c = 0; c < kClusterMax; ++c)  // every remote load in flight
        v[c] = c < cs ? cluster.map_shared_rank(S.hist, c)[tid] : 0;
#pragma unroll
      for (int c = 0; c < kClusterMax; ++c) {
        total += v[c];
        below += c < rank ? v[c] : 0;
      }
      int incl = total;  // inclusive scan of totals over digits (8 warps)
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += u;
      }
      if (lane == 31) S.wsum[warp] = incl;
      S.goff[tid] = incl - total + below;
    }
    __syncthreads();
    if (tid < 256) {
      int add = 0;
      for (int w = 0; w < warp; ++w) add += S.wsum[w];
      S.goff[tid] += add;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kCItems; ++j) {
      const bool valid = base + cpos<ITEMS>(warp, j, lane) < n;
      if (!valid) continue;
      const int digit = (int)((key[j] >> shift) & 255);
      const int r = S.goff[digit] + wc[digit] + rk[j];
      // r < n by construction; the check keeps a corrupted count from
      // addressing a CTA outside the cluster
      if (r >= 0 && r < n) {
        Smem* dst = cluster.map_shared_rank(&S, r / kCTile);
        dst->keys[r % kCTile] = key[j];
        dst->vals[r % kCTile] = val[j];
      }
    }
    cluster.sync();  // every scatter landed
#pragma unroll
    for (int j = 0; j < kCItems; ++j) {
      key[j] = S.keys[cpos<ITEMS>(warp, j, lane)];
      val[j] = S.vals[cpos<ITEMS>(warp, j, lane)];
    }
  }

  // 4. sorted keys and indices out; per level the members before each
  // position (member_count + member_prefix of the multi-launch path)
#pragma unroll
  for (int j = 0; j < kCItems; ++j) {
    const int i = base + cpos<ITEMS>(warp, j, lane);
    if (i < n) {
      keys_out[d.p0 + i] = key[j];
      vals_out[d.p0 + i] = val[j];
    }
  }
  if (levels > 1) {
    for (int l = 1; l < kMaxLevels; ++l) {
      int run = 0;
#pragma unroll
      for (int j = 0; j < kCItems; ++j) {
        const bool m = l < levels && base + cpos<ITEMS>(warp, j, lane) < n &&
                       val[j] < level_size(n, l);
        run += __popc(__ballot_sync(kFull, m));
      }
      if (lane == 0) S.wmem[warp][l] = run;
    }
    __syncthreads();
    if (tid >= 1 && tid < kMaxLevels) {  // exclusive scan over the warps
      int run = 0;
      for (int w = 0; w < kCWarps; ++w) {
        const int c = S.wmem[w][tid];
        S.wmem[w][tid] = run;
        run += c;
      }
      S.lcnt[tid] = run;
    }
    cluster.sync();  // tile totals visible to the cluster
    for (int l = 1; l < kMaxLevels; ++l) {
      if (l >= levels) break;
      int run = S.wmem[warp][l];
#pragma unroll
      for (int c = 0; c < kClusterMax; ++c)  // every remote load in flight
        run += c < rank ? cluster.map_shared_rank(S.lcnt, c)[l] : 0;
#pragma unroll
      for (int j = 0; j < kCItems; ++j) {
        const int i = base + cpos<ITEMS>(warp, j, lane);
        const bool m = i < n && val[j] < level_size(n, l);
        const unsigned bal = __ballot_sync(kFull, m);
        if (i < n) pref[(size_t)(l - 1) * N + d.p0 + i] = run + __popc(bal & lt);
        run += __popc(bal);
      }
    }
  }
  cluster.sync();  // no CTA leaves while another may read its shared memory
}

// ---------------------------------------------------------------------------
// Karras (2012) binary radix tree over sorted keys made unique by their
// position.  Internal node i covers sorted positions [first, last]; its
// children are gamma and gamma+1 (a single position is a point).
__device__ __forceinline__ int common_prefix(const uint64_t* k, int n, int i,
                                             int j) {
  if (j < 0 || j >= n) return -1;
  uint64_t a = k[i], c = k[j];
  if (a != c) return __clzll(a ^ c);
  return 64 + __clz(i ^ j);
}

// Each internal node i > L points ("kept") emits a leaf record for every
// child holding <= L points: (tree, first, last, compact(i)*2 + side); a tree of at most
// L points emits one root record (tree, 0, n-1, -1).  Kept nodes whose two
// children are leaves are listed as climb starts.  Lists are appended with
// one atomic per warp.
template <typename T>
__device__ __forceinline__ void emit(bool want, T rec, T* list, int* count) {
  unsigned mask = __ballot_sync(kFull, want);
  if (!mask) return;
  int lane = threadIdx.x & 31;
  int leader = __ffs(mask) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(count, __popc(mask));
  base = __shfl_sync(kFull, base, leader);
  if (want) list[base + __popc(mask & ((1u << lane) - 1u))] = rec;
}

// Arrival counters start at the number of leaf children (leaves are complete
// before any climb starts); a node with two leaf children starts a climb and
// never receives an arrival.
//
// A node is kept exactly when its range reaches `leaf` positions past i in
// its direction: the common prefix with a key k positions away only shrinks
// as k grows, so one comparison at distance `leaf` decides it.  Each block
// first tests its nodes that way and lists its kept nodes (about one in ten)
// in shared memory; its warps then run the range, split and record work on
// the list only, so the long binary searches of high nodes run on dense
// warps instead of one lane in ten.
//
// Kept nodes get compact indices (one atomic per block on the tree's kept
// count) that address the stored node entries; a kept node beyond the tree's
// capacity sets the tree's overflow flag instead.  Parent links hold the
// parent's radix-tree index (for the arrival counters) and compact index.
__global__ void __launch_bounds__(256)
    karras_kernel(const TreeDesc* desc, const uint64_t* keys, int2* parent,
                  int* counter, int leaf, int4* leaves, int* leaf_count,
                  int2* starts, int* start_count, int* ovf) {
  __shared__ int kept[256];
  __shared__ int nkept, kbase;
  const int b = blockIdx.y;
  const TreeDesc d = desc[b];
  const int n = d.n;
  const uint64_t* k = keys + d.p0;
  int2* par = parent + (d.p0 - b);
  int* cnt = counter + (d.p0 - b);
  int* kept_count = ovf + gridDim.y;
  if (threadIdx.x == 0) nkept = 0;
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  emit(i == 0 && n <= leaf, make_int4(b, 0, n - 1, -1), leaves + d.p0,
       leaf_count + b);
  if (i < n - 1) {
    const int dir =
        common_prefix(k, n, i, i + 1) > common_prefix(k, n, i, i - 1) ? 1 : -1;
    const int dmin = common_prefix(k, n, i, i - dir);
    if (common_prefix(k, n, i, i + leaf * dir) > dmin)
      kept[atomicAdd(&nkept, 1)] = (i << 1) | (dir > 0);
    else
      cnt[i] = 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) kbase = nkept ? atomicAdd(kept_count + b, nkept) : 0;
  __syncthreads();
  const int total = nkept;
  const int lane = threadIdx.x & 31;
  // smallest power of two above `leaf`: every kept range reaches it
  const int lstart = 1 << (32 - __clz(leaf));
  for (int k0 = threadIdx.x & ~31; k0 < total; k0 += blockDim.x) {
    const int ci = kbase + k0 + lane;  // this kept node's compact index
    const bool act = k0 + lane < total && ci < d.cap;
    if (k0 + lane < total && ci >= d.cap) ovf[b] = 1;
    int node = 0;
    bool want0 = false, want1 = false;
    int4 rec0 = make_int4(0, 0, 0, 0), rec1 = rec0;
    if (act) {
      const int e = kept[k0 + lane];
      node = e >> 1;
      const int dir = (e & 1) ? 1 : -1;
      const int dmin = common_prefix(k, n, node, node - dir);
      int lmax = lstart;
      while (common_prefix(k, n, node, node + lmax * dir) > dmin) lmax <<= 1;
      int l = 0;
      for (int t = lmax >> 1; t >= 1; t >>= 1)
        if (common_prefix(k, n, node, node + (l + t) * dir) > dmin) l += t;
      const int j = node + l * dir;
      const int first = min(node, j), last = max(node, j);
      const int dnode = common_prefix(k, n, node, j);
      int s = 0, t = l;
      do {
        t = (t + 1) >> 1;
        if (common_prefix(k, n, node, node + (s + t) * dir) > dnode) s += t;
      } while (t > 1);
      const int gamma = node + s * dir + min(dir, 0);
      if (first != gamma) par[gamma] = make_int2((node << 1) | 0, ci);
      if (last != gamma + 1) par[gamma + 1] = make_int2((node << 1) | 1, ci);
      want0 = gamma - first + 1 <= leaf;
      want1 = last - gamma <= leaf;
      // leaf records name the owner's slot by compact index
      rec0 = make_int4(b, first, gamma, (ci << 1) | 0);
      rec1 = make_int4(b, gamma + 1, last, (ci << 1) | 1);
      cnt[node] = (int)want0 + (int)want1;
    }
    emit(want0, rec0, leaves + d.p0, leaf_count + b);
    emit(want1, rec1, leaves + d.p0, leaf_count + b);
    emit(act && want0 && want1, make_int2(node, ci), starts + (d.p0 - b),
         start_count + b);
  }
}

// ---------------------------------------------------------------------------
struct RefitArgs {
  const TreeDesc* desc;
  const float* x;
  const int* perm;  // sorted local point indices
  const int2* parent;  // per radix-tree node: (parent*2 + side, parent's compact index)
  int* counter;
  const int* pref;  // [level-1][N]: level members before a leaf-order position
  const int4* leaves;
  const int* leaf_count;
  const int2* starts;  // per tree: nodes with two leaf children (index, compact)
  const int* start_count;
  const int* ovf;      // per tree: capacity overflow (tree not refitted)
  float4* pts;
  float4* lpts;
  int* qorder;
  int* wrank;
  Entry* nodes;
  Entry* root;
  int levels;
  int leaf;  // level leaves hold at most this many members
  int N;
};

// Level-leaf reference of `count` members starting at member `start`.
__device__ __forceinline__ int level_leaf_ref(int start, int count) {
  return count > 0 ? leaf_ref(start, count) : kEmptyLeaf;
}

__device__ __forceinline__ Entry* node_entry(Entry* nodes, const TreeDesc& d,
                                             int level, int node, int slot) {
  return nodes + d.node0 + ((size_t)level * d.cap + node) * 2 + slot;
}

__device__ __forceinline__ Entry load_entry_cg(const Entry* e) {
  const float4* p = reinterpret_cast<const float4*>(e);
  float4 a = __ldcg(p), b = __ldcg(p + 1);
  Entry r;
  r.lox = a.x; r.loy = a.y; r.loz = a.z; r.minid = __float_as_int(a.w);
  r.hix = b.x; r.hiy = b.y; r.hiz = b.z; r.ref = __float_as_int(b.w);
  return r;
}

// Arrival counter increment with acquire-release semantics at device scope:
// the caller's earlier node-entry stores are visible to whichever thread
// later observes the incremented count, and that thread sees the sibling's
// stores, without full memory fences.
__device__ __forceinline__ int arrive(int* p) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;"
               : "=r"(old)
               : "l"(p)
               : "memory");
  return old;
}

// Bottom-up climb from completed node i, by one thread: order the two child
// entries by minimum ID (the same order on every level), write their union
// into the parent's slot, and continue while this thread is the second child
// to arrive.  On levels l >= 1 the node becomes a level leaf when both
// children are level leaves holding at most `leaf` members together: the
// members of a subtree are contiguous in the level's member array, the left
// child's (slot 0 until this node swaps) first.
__device__ void climb(const RefitArgs& a, const TreeDesc& d, int b, int i,
                      int ci) {
  const int2* par = a.parent + (d.p0 - b);
  int* cnt = a.counter + (d.p0 - b);
  // i: the node's radix-tree index (parent links, arrival counters); ci: its
  // compact index (stored entries).  Karras depth is below 97 (64 key bits +
  // 32 index bits); the bound only guards against a corrupted topology.
  for (int step = 0; step < 128; ++step) {
    // issue every level's loads before any store (one L2 round trip)
    Entry u[kMaxLevels], v[kMaxLevels];
#pragma unroll
    for (int l = 0; l < kMaxLevels; ++l) {
      if (l < a.levels) {
        u[l] = load_entry_cg(node_entry(a.nodes, d, l, ci, 0));
        v[l] = load_entry_cg(node_entry(a.nodes, d, l, ci, 1));
      }
    }
    const int2 pc = i ? par[i] : make_int2(0, 0);
    bool swap = v[0].minid < u[0].minid;
#pragma unroll
    for (int l = 0; l < kMaxLevels; ++l) {
      if (l >= a.levels) break;
      if (swap) {
        store_entry(node_entry(a.nodes, d, l, ci, 0), v[l]);
        store_entry(node_entry(a.nodes, d, l, ci, 1), u[l]);
      }
      Entry e;
      e.lox = fminf(u[l].lox, v[l].lox); e.loy = fminf(u[l].loy, v[l].loy);
      e.loz = fminf(u[l].loz, v[l].loz); e.hix = fmaxf(u[l].hix, v[l].hix);
      e.hiy = fmaxf(u[l].hiy, v[l].hiy); e.hiz = fmaxf(u[l].hiz, v[l].hiz);
      e.minid = min(u[l].minid, v[l].minid);
      e.ref = ci;
      if (l > 0 && u[l].ref < 0 && v[l].ref < 0) {
        int cu = level_leaf_count(u[l].ref), cv = level_leaf_count(v[l].ref);
        if (cu + cv <= a.leaf) {
          int su = 0, sv = 0, k;
          if (cu) leaf_decode(u[l].ref, su, k);
          if (cv) leaf_decode(v[l].ref, sv, k);
          e.ref = level_leaf_ref(cu ? su : sv, cu + cv);
        }
      }
      if (i == 0)
        a.root[b * a.levels + l] = e;
      else
        store_entry(node_entry(a.nodes, d, l, pc.y, pc.x & 1), e);
    }
    if (i == 0 || arrive(cnt + (pc.x >> 1)) == 0) return;
    i = pc.x >> 1;
    ci = pc.y;
  }
}

// Groups of G lanes (G = 16 for leaves of up to 16 points, else 32) each take
// one leaf record: lane k takes sorted position first + k, ranks its
// original ID among the leaf's IDs and writes pts in ascending ID order; per
// level, redux.sync min/max over order-preserving integer keys give the box
// of the finite members with ID < n/4^l; the group's first lane writes the
// entries into the owner node's slot (or the root).  The members of level l
// are the leaf's first ranks; they go to the level's query order and member
// array from the leaf's member offset `pref`, which is also the start of the
// level-l leaf reference.  Two groups per warp keep twice as many leaves in
// flight; no arrivals here -- the counters were initialised with the
// leaf-child counts.
// Eight resident CTAs per SM (32 registers, a few spilled): the kernel is
// issue bound at low occupancy, 64 rooms 96 -> 85 us under ncu.
template <int G>
__global__ void __launch_bounds__(256, 8) leaf_kernel(RefitArgs a) {
  int lane = threadIdx.x & 31;
  int gl = lane & (G - 1);
  unsigned gmask = G == 32 ? kFull : (0xffffu << (lane & 16));
  int group = (blockIdx.x * blockDim.x + threadIdx.x) / G;
  int groups = (gridDim.x * blockDim.x) / G;
  const int b = blockIdx.y;
  const TreeDesc d = a.desc[b];
  if (a.ovf[b]) return;  // kept nodes beyond capacity: the tree is not used
  int total = a.leaf_count[b];
  const float inf = __int_as_float(0x7f800000);
  for (int r = group; r < total; r += groups) {
    int4 rec = a.leaves[d.p0 + r];
    int cf = rec.y, c = rec.z - rec.y + 1, code = rec.w;
    bool on = gl < c;
    // the leaf's member offset on level l (lane l loads it; level 0: cf),
    // issued together with the point loads
    int st = cf;
    if (gl >= 1 && gl < a.levels)
      st = __ldcg(a.pref + (size_t)(gl - 1) * a.N + d.p0 + cf);
    int id = on ? a.perm[d.p0 + cf + gl] : INT_MAX;
    float px = 0.f, py = 0.f, pz = 0.f;
    if (on) {
      const float* p = a.x + 3ll * (d.p0 + id);
      px = p[0];
      py = p[1];
      pz = p[2];
    }
    // lanes past the leaf's count hold INT_MAX, so a fixed G-step loop ranks
    // without diverging between the two half-warp groups of a warp
    int rank = 0;
#pragma unroll
    for (int j = 0; j < G; ++j) rank += __shfl_sync(gmask, id, j, G) < id;
    if (on) a.pts[d.p0 + cf + rank] = make_float4(px, py, pz, __int_as_float(id));
    int minid = (int)__reduce_min_sync(gmask, (unsigned)id);
    bool fin = on && finite3(px, py, pz);
    unsigned kx = float_key(px), ky = float_key(py), kz = float_key(pz);
    Entry* own = code < 0 ? nullptr : node_entry(a.nodes, d, 0, code >> 1, code & 1);
    int* qo = a.qorder + d.q0;           // level 0 of this tree's query order
    float4* lp = a.lpts + (d.q0 - d.p0);  // level 1 of its member arrays
#pragma unroll
    for (int l = 0; l < kMaxLevels; ++l) {
      if (l >= a.levels) break;
      bool mem = on && id < level_size(d.n, l);
      int members = __popc(__ballot_sync(gmask, mem));
      int start = __shfl_sync(gmask, st, l, G);
      if (mem) {
        qo[start + rank] = id;
        if (l) lp[start + rank] = make_float4(px, py, pz, __int_as_float(id));
      }
      // members before this point in leaf order (the leaf's members first)
      if (on)
        a.wrank[(size_t)(d.p0 + id) * a.levels + l] = start + min(rank, members);
      qo += level_size(d.n, l);
      if (l) lp += level_size(d.n, l);
      bool f = mem && fin;
      Entry t;
      t.lox = t.loy = t.loz = inf;
      t.hix = t.hiy = t.hiz = -inf;
      if (__ballot_sync(gmask, f)) {
        t.lox = key_float(__reduce_min_sync(gmask, f ? kx : 0xffffffffu));
        t.loy = key_float(__reduce_min_sync(gmask, f ? ky : 0xffffffffu));
        t.loz = key_float(__reduce_min_sync(gmask, f ? kz : 0xffffffffu));
        t.hix = key_float(__reduce_max_sync(gmask, f ? kx : 0u));
        t.hiy = key_float(__reduce_max_sync(gmask, f ? ky : 0u));
        t.hiz = key_float(__reduce_max_sync(gmask, f ? kz : 0u));
      }
      t.minid = minid;
      t.ref = level_leaf_ref(start, members);
      if (gl == 0) {
        if (own)
          store_entry(own + (size_t)l * d.cap * 2, t);
        else
          a.root[b * a.levels + l] = t;
      }
    }
  }
}

// One thread per listed climb start (nodes whose two children are leaves; a
// tree's list is about a third of its leaf count).  Climbs run as
// independent threads, so every path of every tree proceeds at once and a
// tree's refit takes about its depth in steps; launching only the starts
// keeps every climbing thread resident from the first step.
__global__ void __launch_bounds__(256) climb_kernel(RefitArgs a) {
  int b = blockIdx.y;
  TreeDesc d = a.desc[b];
  if (a.ovf[b]) return;
  const int2* st = a.starts + (d.p0 - b);
  int total = a.start_count[b];
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < total;
       r += gridDim.x * blockDim.x)
    climb(a, d, b, st[r].x, st[r].y);
}

// One warp per (level, tree): the top of the level's tree expanded breadth
// first while the list still fits 32 entries, stopping at the level's
// leaves.  The list covers every point of the level exactly once, so a
// frontier walk may start from it (one step of independent entry loads)
// instead of descending from the root one dependent step per level.
__global__ void __launch_bounds__(32) cut_kernel(const TreeDesc* desc,
                                                 const Entry* nodes,
                                                 const Entry* root,
                                                 int levels, int* cut,
                                                 const int* ovf) {
  constexpr int CH = kCutMax / 32;  // list items per lane: c * 32 + lane
  __shared__ int next[kCutMax];
  const int l = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
  if (ovf[b]) return;  // the tree is not used
  const TreeDesc d = desc[b];
  const Entry* nl = nodes + d.node0 + (size_t)l * d.cap * 2;
  const unsigned lt = (1u << lane) - 1u;
  const int rref = root[b * levels + l].ref;
  int cnt = 1;
  int ei[CH], ref[CH];  // item c * 32 + lane < cnt: entry (-1: the root), ref
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    ei[c] = -1;
    ref[c] = (c == 0 && lane == 0) ? rref : -1;
  }
  // each step grows the list by at least one, so at most kCutMax-1 steps
  for (int step = 0; step < kCutMax; ++step) {
    unsigned bi[CH];
    int grown = cnt, before = 0;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      bi[c] = __ballot_sync(kFull, c * 32 + lane < cnt && ref[c] >= 0);
      grown += __popc(bi[c]);
    }
    if (grown == cnt || grown > kCutMax) break;
    // in list order: a leaf keeps one slot, an internal node becomes its
    // two children
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int item = c * 32 + lane;
      const int pos = item + before + __popc(bi[c] & lt);
      if (item < cnt) {
        if ((bi[c] >> lane) & 1u) {
          next[pos] = 2 * ref[c];
          next[pos + 1] = 2 * ref[c] + 1;
        } else {
          next[pos] = ei[c];
        }
      }
      before += __popc(bi[c]);
    }
    __syncwarp();
    cnt = grown;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int item = c * 32 + lane;
      ei[c] = item < cnt ? next[item] : -1;
      ref[c] = item < cnt ? (ei[c] >= 0 ? load_entry(nl + ei[c]).ref : rref) : -1;
    }
    __syncwarp();
  }
  int* out = cut + ((size_t)b * levels + l) * kCutStride;
  if (lane == 0) out[0] = cnt;
#pragma unroll
  for (int c = 0; c < CH; ++c)
    if (c * 32 + lane < cnt) out[1 + c * 32 + lane] = ei[c];
}

// ---------------------------------------------------------------------------
// Members of levels 1.. (IDs < n/4^l) before every sorted position: a tile
// count, an exclusive scan over (level, tile) and a per-tile scan.  Leaves
// keep their sorted point range, so these are also the counts before every
// leaf-order position.  Counter layout per tree:
// cnt[(tree*(levels-1) + level-1)*max_tiles + tile].
__global__ void __launch_bounds__(kSortThreads)
    member_count(const TreeDesc* desc, const int* ids, int levels, int* cnt,
                 int max_tiles) {
  __shared__ int h[kMaxLevels];
  TreeDesc d = desc[blockIdx.y];
  int base = blockIdx.x * kSortTile;
  if (base >= d.n) return;
  if (threadIdx.x < kMaxLevels) h[threadIdx.x] = 0;
  __syncthreads();
  int c[kMaxLevels] = {0, 0, 0, 0};
  for (int j = 0; j < kSortItems; ++j) {
    int idx = base + j * kSortThreads + threadIdx.x;
    if (idx < d.n) {
      int id = ids[d.p0 + idx];
      for (int l = 1; l < levels; ++l) c[l] += id < level_size(d.n, l);
    }
  }
  for (int l = 1; l < levels; ++l) {
    int v = c[l];
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    if ((threadIdx.x & 31) == 0) atomicAdd(&h[l], v);
  }
  __syncthreads();
  int l = threadIdx.x + 1;
  if (l < levels)
    cnt[((size_t)blockIdx.y * (levels - 1) + l - 1) * max_tiles + blockIdx.x] =
        h[l];
}

__global__ void __launch_bounds__(kSortThreads)
    member_prefix(const TreeDesc* desc, const int* ids, int levels,
                  const int* cnt, int max_tiles, int* pref, int N) {
  __shared__ int run[kMaxLevels];
  __shared__ int wsum[kSortThreads / 32][kMaxLevels];
  TreeDesc d = desc[blockIdx.y];
  int base = blockIdx.x * kSortTile;
  if (base >= d.n) return;
  int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid + 1 < levels)
    run[tid + 1] =
        cnt[((size_t)blockIdx.y * (levels - 1) + tid) * max_tiles + blockIdx.x];
  __syncthreads();
  int idv[kSortItems];
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    int idx = base + j * kSortThreads + tid;
    idv[j] = idx < d.n ? ids[d.p0 + idx] : INT_MAX;
  }
#pragma unroll
  for (int j = 0; j < kSortItems; ++j) {
    int idx = base + j * kSortThreads + tid;
    int id = idv[j];
    unsigned bal[kMaxLevels];
#pragma unroll
    for (int l = 1; l < kMaxLevels; ++l) {
      if (l >= levels) break;
      bal[l] = __ballot_sync(kFull, id < level_size(d.n, l));
      if (lane == 0) wsum[warp][l] = __popc(bal[l]);
    }
    __syncthreads();
    // the scan runs over levels 1.. in turn: `start` is level l's first slot
    int start = 0;
#pragma unroll
    for (int l = 1; l < kMaxLevels; ++l) {
      if (l >= levels) break;
      int r = run[l] + __popc(bal[l] & ((1u << lane) - 1u));
      for (int w = 0; w < warp; ++w) r += wsum[w][l];
      if (idx < d.n) pref[(size_t)(l - 1) * N + d.p0 + idx] = r - start;
      start += level_size(d.n, l);
    }
    __syncthreads();
    if (tid >= 1 && tid < levels) {
      int s = 0;
      for (int w = 0; w < kSortThreads / 32; ++w) s += wsum[w][tid];
      run[tid] += s;
    }
    __syncthreads();
  }
}

inline int blocks_for(long long n, int per) {
  return (int)std::max<long long>(1, (n + per - 1) / per);
}

// Blocks per tree of the climb kernel: one thread per 16 points, above the
// usual start count (about n / 20 with leaves of ~10 points); threads loop
// over any excess.
int climb_grid(long long max_points) { return blocks_for((max_points + 15) / 16, 256); }

// Blocks per tree of the leaf kernel (grid.y = tree): enough lane groups for
// one leaf record per 8 points (leaves hold about 10 points on average; the
// groups loop over any excess), never more than the largest tree can use.
int leaf_grid(bool half_warps, long long max_points) {
  long long groups_per_block = half_warps ? 16 : 8;
  long long records = (max_points + 7) / 8;
  return (int)std::max<long long>(1, (records + groups_per_block - 1) / groups_per_block);
}

}  // namespace

// Build temporaries.  A forest made by build_forest frees them when the
// build is enqueued; rebuild_forest keeps them with the forest, so that later
// rebuilds of the same shape allocate nothing (and can be captured in a CUDA
// graph).
struct BuildScratch {
  uint64_t* keys = nullptr;
  uint64_t* keys2 = nullptr;
  int* vals = nullptr;
  int* vals2 = nullptr;
  int* hist = nullptr;
  unsigned* bounds = nullptr;
  int4* leaves = nullptr;  // leaf records; at most one per point
  int2* parent = nullptr;  // per radix-tree node: (parent*2 + side, parent's compact index)
  int* counter = nullptr;  // arrival counters + leaf-record and climb-start counts
  int* pref = nullptr;
  int2* starts = nullptr;  // climb starts: (radix-tree index, compact index)
  void* block = nullptr;   // the one pool allocation holding all of the above
};

namespace {

// Sub-buffers of one pool allocation, each on a 256-byte boundary: a build
// allocates its forest and its temporaries with one call each (and frees the
// temporaries with one), instead of one native-pool call per array, which
// took tens of microseconds of host time per build.
class Carve {
 public:
  template <typename T>
  void add(T** p, long long count) {
    const size_t n = sizeof(T) * (size_t)std::max<long long>(count, 1);
    slots_[used_] = reinterpret_cast<void**>(p);
    offs_[used_++] = bytes_;
    bytes_ += (n + 255) & ~size_t(255);
  }
  cudaError_t alloc(void** block, cudaStream_t s) {
    cudaError_t e = pool_alloc(block, bytes_, s);
    if (e) return e;
    for (int i = 0; i < used_; ++i)
      *slots_[i] = static_cast<char*>(*block) + offs_[i];
    return cudaSuccess;
  }

 private:
  void** slots_[16];
  size_t offs_[16];
  int used_ = 0;
  size_t bytes_ = 0;
};

int max_tiles_of(const Forest* f) { return blocks_for(f->max_n, kSortTile); }

long long inner_nodes(const Forest* f) { return std::max<long long>(1, (long long)f->N - f->B); }

// Every tree is keyed and sorted by one cluster launch (else the
// multi-launch sort, which needs the double buffers and digit histograms).
bool cluster_path(const Forest* f) {
  return GSA_CLUSTER_SORT && f->max_n <= kClusterMaxPoints;
}

cudaError_t alloc_scratch(const Forest* f, BuildScratch* sc, cudaStream_t s) {
  const long long N = f->N, B = f->B, inner = inner_nodes(f);
  Carve c;
  c.add(&sc->pref, (f->levels - 1) * N);
  c.add(&sc->starts, inner);
  c.add(&sc->vals, N);
  c.add(&sc->keys, N);
  if (!cluster_path(f)) {
    c.add(&sc->keys2, N);
    c.add(&sc->vals2, N);
    c.add(&sc->hist, 256ll * B * max_tiles_of(f));
  }
  c.add(&sc->bounds, 6 * B);
  c.add(&sc->leaves, N);
  c.add(&sc->parent, inner);
  c.add(&sc->counter, inner + 2 * B);
  return c.alloc(&sc->block, s);
}

cudaError_t free_scratch(BuildScratch* sc, cudaStream_t s) {
  cudaError_t e = pool_free(sc->block, s);
  *sc = BuildScratch();
  return e;
}

template <int ITEMS, int MINB>
cudaError_t launch_cluster_sort_items(const Forest* f, const float* x,
                                      const BuildScratch& sc, cudaStream_t s) {
  static std::atomic<unsigned long long> attr_set{0};  // one bit per device
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e) return e;
  const unsigned long long bit = 1ull << (device & 63);
  if (!(attr_set.load(std::memory_order_relaxed) & bit)) {
    e = cudaFuncSetAttribute(cluster_sort_kernel<ITEMS, MINB>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(ClusterSmem<ITEMS>));
    // clusters above the portable size of 8
    if (!e)
      e = cudaFuncSetAttribute(cluster_sort_kernel<ITEMS, MINB>,
                               cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e) return e;
    attr_set.fetch_or(bit, std::memory_order_relaxed);
  }
  const int cs = blocks_for(f->max_n, kCThreads * ITEMS);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, f->B);
  cfg.blockDim = dim3(kCThreads);
  cfg.dynamicSmemBytes = sizeof(ClusterSmem<ITEMS>);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, cluster_sort_kernel<ITEMS, MINB>, f->desc, x,
                            morton_bits(f->max_n), f->levels, sc.keys,
                            sc.vals, sc.pref, f->N);
}

// Very few trees (their 4,096-position tiles would fill at most an eighth of
// the SMs, e.g. the session's one tree per build): tiles of 2,048 in
// clusters of up to 16, so each CTA ranks half as many items per pass (one
// 24,000-point tree: build 125 -> 111 us); otherwise tiles of 4,096 in
// portable clusters of up to 8 (8 trees: 144 us, against 158 us with the
// 16-CTA clusters, which the GPCs place less freely), with the register
// budget of three CTAs per SM once two per SM would take a second wave (64
// rooms: 152 -> 130 us under ncu; fewer tiles keep 64 registers, since the
// spills only add latency when the tiles fit anyway).
cudaError_t launch_cluster_sort(const Forest* f, const float* x,
                                const BuildScratch& sc, cudaStream_t s) {
  int device = 0, sms = 148;
  if (cudaGetDevice(&device) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const long long ctas = (long long)f->B * blocks_for(f->max_n, kCThreads * 8);
  if (GSA_SMALL_SORT_TILES && 8 * ctas <= sms)
    return launch_cluster_sort_items<4, 1>(f, x, sc, s);
  if (ctas > 2ll * sms) return launch_cluster_sort_items<8, 3>(f, x, sc, s);
  return launch_cluster_sort_items<8, 2>(f, x, sc, s);
}

// Enqueues every build kernel of `f` over points `x` (the layout in f->hdesc)
// using the temporaries in `sc`.  Allocates nothing.
cudaError_t enqueue_build(Forest* f, const float* x, const BuildScratch& sc,
                          cudaStream_t s) {
  const int B = f->B, max_n = f->max_n;
  const long long N = f->N, inner = inner_nodes(f);
  const int max_tiles = max_tiles_of(f);
  uint64_t *keys = sc.keys, *keys2 = sc.keys2;
  int *vals = sc.vals, *vals2 = sc.vals2, *hist = sc.hist;
  int* counter = sc.counter;
  cudaError_t e = cudaMemsetAsync(counter, 0, sizeof(int) * (inner + 2 * B), s);
  if (!e) e = cudaMemsetAsync(f->ovf, 0, sizeof(int) * 2 * B, s);
  if (e) return e;
  int* leaf_count = counter + inner;
  int* start_count = leaf_count + B;

  for (int b0 = 0; b0 < B; b0 += 256) {
    DescChunk c;
    c.first = b0;
    c.count = std::min(256, B - b0);
    for (int i = 0; i < c.count; ++i) c.d[i] = f->hdesc[b0 + i];
    upload_desc<<<1, 256, 0, s>>>(f->desc, c, sc.bounds);
  }
  int launches = (B + 255) / 256;
  dim3 gs(max_tiles, B);
  dim3 gk(blocks_for(std::max(1, max_n - 1), 256), B);
  if (cluster_path(f)) {
    // one cluster per tree: bounds, keys, sort and member offsets
    e = launch_cluster_sort(f, x, sc, s);
    if (e) return e;
    karras_kernel<<<gk, 256, 0, s>>>(f->desc, sc.keys, sc.parent, counter,
                                     f->leaf, sc.leaves, leaf_count, sc.starts,
                                     start_count, f->ovf);
    launches += 2;
  } else {
    dim3 g(std::min(blocks_for(max_n, 1024), 64), B);
    bounds_kernel<<<g, 256, 0, s>>>(f->desc, x, sc.bounds);
    dim3 gm(std::min(blocks_for(max_n, 256 * kUnroll), 1024), B);
    const int bits = morton_bits(max_n);
    const int passes = (3 * bits + 7) / 8;
    morton_kernel<<<gm, 256, 0, s>>>(f->desc, x, sc.bounds, bits, keys, vals);
    for (int pass = 0; pass < passes; ++pass) {
      int shift = 8 * pass;
      sort_upsweep<<<gs, kSortThreads, 0, s>>>(f->desc, keys, shift, hist,
                                               max_tiles);
      seg_scan<<<B, kScanThreads, 0, s>>>(f->desc, hist, 256, max_tiles,
                                          kSortTile);
      sort_scatter<<<gs, kSortThreads, 0, s>>>(f->desc, keys, vals, keys2,
                                               vals2, hist, shift, max_tiles);
      std::swap(keys, keys2);
      std::swap(vals, vals2);
    }
    karras_kernel<<<gk, 256, 0, s>>>(f->desc, keys, sc.parent, counter,
                                     f->leaf, sc.leaves, leaf_count, sc.starts,
                                     start_count, f->ovf);
    launches += 2 + 3 * passes + 1;
    if (f->levels > 1) {
      // members of each prefix level before every sorted position
      member_count<<<gs, kSortThreads, 0, s>>>(f->desc, vals, f->levels, hist,
                                               max_tiles);
      seg_scan<<<B, kScanThreads, 0, s>>>(f->desc, hist, f->levels - 1,
                                          max_tiles, kSortTile);
      member_prefix<<<gs, kSortThreads, 0, s>>>(f->desc, vals, f->levels, hist,
                                                max_tiles, sc.pref, (int)N);
      launches += 3;
    }
  }
  RefitArgs ra;
  ra.desc = f->desc;
  ra.x = x;
  ra.perm = vals;
  ra.parent = sc.parent;
  ra.counter = counter;
  ra.pref = sc.pref;
  ra.leaves = sc.leaves;
  ra.leaf_count = leaf_count;
  ra.starts = sc.starts;
  ra.start_count = start_count;
  ra.ovf = f->ovf;
  ra.pts = f->pts;
  ra.lpts = f->lpts;
  ra.qorder = f->qorder;
  ra.wrank = f->wrank;
  ra.nodes = f->nodes;
  ra.root = f->root;
  ra.levels = f->levels;
  ra.leaf = f->leaf;
  ra.N = (int)N;
  // lane groups of each tree loop over its leaf records (their count is
  // only known on the device)
  dim3 gl(leaf_grid(f->leaf <= 16, max_n), B);
  if (f->leaf <= 16)
    leaf_kernel<16><<<gl, 256, 0, s>>>(ra);
  else
    leaf_kernel<32><<<gl, 256, 0, s>>>(ra);
  climb_kernel<<<dim3(climb_grid(max_n), B), 256, 0, s>>>(ra);
  cut_kernel<<<dim3(f->levels, B), 32, 0, s>>>(f->desc, f->nodes, f->root,
                                               f->levels, f->cut, f->ovf);
  launches += 3;
  count_launches(launches);
  return cudaGetLastError();
}

}  // namespace

cudaError_t sort_query_rows(const float* q, int n, const int** perm,
                            void** block, cudaStream_t s) {
  *perm = nullptr;
  *block = nullptr;
  if (!q || n < 1 || n > kMaxPoints) return cudaErrorInvalidValue;
  // the queries laid out as one tree whose build stops after the key sort
  Forest f;
  f.B = 1;
  f.levels = 1;
  f.N = n;
  f.max_n = n;
  f.hdesc.resize(1);
  f.hdesc[0].p0 = 0;
  f.hdesc[0].n = n;
  f.hdesc[0].node0 = 0;
  f.hdesc[0].q0 = 0;
  f.hdesc[0].cap = 0;
  BuildScratch sc;
  const bool cluster = cluster_path(&f);
  Carve c;
  c.add(&f.desc, 1);
  c.add(&sc.keys, n);
  c.add(&sc.vals, n);
  c.add(&sc.bounds, 6);
  if (!cluster) {
    c.add(&sc.keys2, n);
    c.add(&sc.vals2, n);
    c.add(&sc.hist, 256ll * max_tiles_of(&f));
  }
  cudaError_t e = c.alloc(block, s);
  if (e) return e;
  DescChunk dc;
  dc.first = 0;
  dc.count = 1;
  dc.d[0] = f.hdesc[0];
  upload_desc<<<1, 256, 0, s>>>(f.desc, dc, sc.bounds);
  int launches = 1;
  const int* order = sc.vals;
  if (cluster) {
    e = launch_cluster_sort(&f, q, sc, s);  // one level: no member offsets
    launches += 1;
  } else {
    uint64_t *keys = sc.keys, *keys2 = sc.keys2;
    int *vals = sc.vals, *vals2 = sc.vals2;
    const int max_tiles = max_tiles_of(&f);
    dim3 gs(max_tiles, 1);
    bounds_kernel<<<dim3(std::min(blocks_for(n, 1024), 64), 1), 256, 0, s>>>(
        f.desc, q, sc.bounds);
    const int bits = morton_bits(n);
    const int passes = (3 * bits + 7) / 8;
    morton_kernel<<<dim3(std::min(blocks_for(n, 256 * kUnroll), 1024), 1), 256,
                    0, s>>>(f.desc, q, sc.bounds, bits, keys, vals);
    for (int pass = 0; pass < passes; ++pass) {
      sort_upsweep<<<gs, kSortThreads, 0, s>>>(f.desc, keys, 8 * pass,
                                               sc.hist, max_tiles);
      seg_scan<<<1, kScanThreads, 0, s>>>(f.desc, sc.hist, 256, max_tiles,
                                          kSortTile);
      sort_scatter<<<gs, kSortThreads, 0, s>>>(f.desc, keys, vals, keys2,
                                               vals2, sc.hist, 8 * pass,
                                               max_tiles);
      std::swap(keys, keys2);
      std::swap(vals, vals2);
    }
    order = vals;
    launches += 2 + 3 * passes;
  }
  count_launches(launches);
  if (!e) e = cudaGetLastError();
  if (!e) *perm = order;
  return e;
}

cudaError_t build_forest(const float* x, const int* seg, int B, int prefix,
                         int leaf, cudaStream_t s, Forest** out) {
  *out = nullptr;
  if (B < 1 || B > 65535 || !x || leaf < 1) return cudaErrorInvalidValue;
  Forest* f = new (std::nothrow) Forest();
  if (!f) return cudaErrorMemoryAllocation;
  f->B = B;
  f->levels = prefix ? kMaxLevels : 1;
  f->leaf = std::min(leaf, kMaxLeaf);
  f->x = x;
  f->hdesc.resize(B);
  long long node_entries = 0, q_total = 0, N = 0;
  int max_n = 0;
  for (int b = 0; b < B; ++b) {
    int n = seg[b + 1] - seg[b];
    if (n < 1 || seg[b] != N) {
      delete f;
      return cudaErrorInvalidValue;
    }
    TreeDesc& d = f->hdesc[b];
    d.p0 = (int)N;
    d.n = n;
    d.node0 = (int)node_entries;
    d.q0 = (int)q_total;
    d.cap = node_capacity(n, f->leaf);
    node_entries += 2ll * f->levels * d.cap;
    for (int l = 0; l < f->levels; ++l) q_total += level_size(n, l);
    N += n;
    max_n = std::max(max_n, n);
  }
  if (N > kMaxPoints || node_entries > INT_MAX || q_total > INT_MAX) {
    delete f;
    return cudaErrorInvalidValue;
  }
  f->N = (int)N;
  f->max_n = max_n;
  f->q_total = q_total;

  Carve c;
  c.add(&f->desc, B);
  c.add(&f->pts, N);
  c.add(&f->nodes, node_entries);
  c.add(&f->root, (long long)B * f->levels);
  c.add(&f->qorder, q_total);
  c.add(&f->lpts, q_total - N);
  c.add(&f->wrank, N * f->levels);
  c.add(&f->cut, (long long)kCutStride * B * f->levels);
  c.add(&f->ovf, 2ll * B);
  cudaError_t e = c.alloc(&f->block, s);
  BuildScratch sc;
  if (!e) e = alloc_scratch(f, &sc, s);
  if (!e) e = enqueue_build(f, x, sc, s);
  cudaError_t fe = free_scratch(&sc, s);
  if (!e) e = fe;
  if (e) {
    free_forest(f, s);
    return e;
  }
  *out = f;
  return cudaSuccess;
}

cudaError_t rebuild_forest(Forest* f, const float* x, cudaStream_t s) {
  if (!f || !x) return cudaErrorInvalidValue;
  if (!f->scratch) {
    BuildScratch* sc = new (std::nothrow) BuildScratch();
    if (!sc) return cudaErrorMemoryAllocation;
    cudaError_t e = alloc_scratch(f, sc, s);
    if (e) {
      free_scratch(sc, s);
      delete sc;
      return e;
    }
    f->scratch = sc;
  }
  f->x = x;
  return enqueue_build(f, x, *f->scratch, s);
}

cudaError_t free_forest(Forest* f, cudaStream_t s) {
  if (!f) return cudaSuccess;
  cudaError_t e = pool_free(f->block, s);
  if (f->scratch) {
    cudaError_t fe = free_scratch(f->scratch, s);
    if (!e) e = fe;
    delete f->scratch;
  }
  delete f;
  return e;
}

}  // namespace gsa
