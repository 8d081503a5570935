// SPDX-License-Identifier: Apache-2.0
// libreference_queries: the original-order brute-force radius and 3NN scans
// that GSA uses for small supports (N <= threshold) and as its exactness
// reference (GSA csrc/reference_queries.cu:6-123, exports `ball`, `nn3`).
//
// Contract kept from the reference kernels:
//  * ball: scan support IDs 0..n-1, collect the first `ns` with
//    d2 < r*r; a row with at least one hit is [hits..., first hit repeated];
//    a row with no hit is left untouched (callers pre-zero it).
//  * nn3: the three smallest finite d2 in (d2, id) order -- a strict `<`
//    during an ascending-ID scan keeps the lower ID on ties; missing entries
//    are (inf, 0).  (The reference compares in double against 1e40, which
//    rejects +inf and NaN exactly like the finite test used here.)
//
// B200 execution: each block owns 256 queries of one batch item and streams
// the support through shared memory in SoA tiles (broadcast reads); radius
// rows are assembled in shared memory and stored row-by-row with coalesced
// warp writes.  The block stops streaming once every query has `ns` hits.
#include <algorithm>
#include "common.cuh"

namespace gsa {
namespace {

constexpr int kThreads = 256;
constexpr int kTile = 1024;
constexpr int kSmemK = 32;

__device__ __forceinline__ void load_tile(const float* x, int base, int count,
                                          float* sx, float* sy, float* sz) {
  for (int i = threadIdx.x; i < count; i += kThreads) {
    const float* p = x + 3ll * (base + i);
    sx[i] = p[0];
    sy[i] = p[1];
    sz[i] = p[2];
  }
}

__global__ void __launch_bounds__(kThreads)
    ball_scan_kernel(int n, int m, float radius, int ns, const float* q,
                     const float* x, int* idx) {
  __shared__ float sx[kTile], sy[kTile], sz[kTile];
  __shared__ int rows[kThreads][kSmemK + 1];
  int bi = blockIdx.y;
  int t = blockIdx.x * kThreads + threadIdx.x;
  bool valid = t < m;
  const float* qb = q + 3ll * m * bi;
  const float* xb = x + 3ll * n * bi;
  int* ob = idx + (long long)m * ns * bi;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (valid) {
    px = qb[3ll * t];
    py = qb[3ll * t + 1];
    pz = qb[3ll * t + 2];
  }
  const float r2 = __fmul_rn(radius, radius);
  const bool in_smem = ns <= kSmemK;
  int* row = rows[threadIdx.x];
  int cnt = 0;
  for (int base = 0; base < n; base += kTile) {
    if (!__syncthreads_or(valid && cnt < ns)) break;
    int c = min(kTile, n - base);
    load_tile(xb, base, c, sx, sy, sz);
    __syncthreads();
    if (valid) {
      for (int k = 0; k < c && cnt < ns; ++k) {
        if (exact_d2(px, py, pz, sx[k], sy[k], sz[k]) < r2) {
          int id = base + k;
          if (in_smem) {
            row[cnt] = id;
          } else {
            int* o = ob + (long long)t * ns;
            if (cnt == 0)
              for (int l = 0; l < ns; ++l) o[l] = id;
            o[cnt] = id;
          }
          ++cnt;
        }
      }
    }
    __syncthreads();
  }
  if (!in_smem) return;
  __syncwarp();
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = 0; j < 32; ++j) {
    int tj = blockIdx.x * kThreads + warp * 32 + j;
    int cj = __shfl_sync(kFull, cnt, j);
    if (tj >= m || cj == 0) continue;
    if (lane < ns) {
      const int* rj = rows[warp * 32 + j];
      ob[(long long)tj * ns + lane] = rj[lane < cj ? lane : 0];
    }
  }
}

__global__ void __launch_bounds__(kThreads)
    nn3_scan_kernel(int n, int m, const float* q, const float* x, float* d,
                    int* idx) {
  __shared__ float sx[kTile], sy[kTile], sz[kTile];
  int bi = blockIdx.y;
  int t = blockIdx.x * kThreads + threadIdx.x;
  bool valid = t < n;
  const float* qb = q + 3ll * n * bi;
  const float* xb = x + 3ll * m * bi;
  float px = 0.f, py = 0.f, pz = 0.f;
  if (valid) {
    px = qb[3ll * t];
    py = qb[3ll * t + 1];
    pz = qb[3ll * t + 2];
  }
  const float inf = __int_as_float(0x7f800000);
  float b0 = inf, b1 = inf, b2 = inf;
  int i0 = 0, i1 = 0, i2 = 0;
  for (int base = 0; base < m; base += kTile) {
    int c = min(kTile, m - base);
    __syncthreads();
    load_tile(xb, base, c, sx, sy, sz);
    __syncthreads();
    if (!valid) continue;
    for (int k = 0; k < c; ++k) {
      float v = exact_d2(px, py, pz, sx[k], sy[k], sz[k]);
      if (v < b2) {  // false for +inf and NaN
        int id = base + k;
        if (v < b1) {
          b2 = b1;
          i2 = i1;
          if (v < b0) {
            b1 = b0;
            i1 = i0;
            b0 = v;
            i0 = id;
          } else {
            b1 = v;
            i1 = id;
          }
        } else {
          b2 = v;
          i2 = id;
        }
      }
    }
  }
  if (valid) {
    long long o = 3ll * n * bi + 3ll * t;
    d[o] = b0;
    d[o + 1] = b1;
    d[o + 2] = b2;
    idx[o] = i0;
    idx[o + 1] = i1;
    idx[o + 2] = i2;
  }
}

}  // namespace
}  // namespace gsa

using namespace gsa;

// See include/reference_queries.h.
GSA_API int ball(int b, int n, int m, float r, int ns, const float* q,
                 const float* x, int* idx, void* s) {
  if (b < 0 || n < 0 || m < 0 || ns < 1) return -2;
  if (!b || !m) return 0;
  if (!q || !idx || (n && !x)) return -2;
  dim3 grid((m + kThreads - 1) / kThreads, b);
  count_launches();
  ball_scan_kernel<<<grid, kThreads, 0, (cudaStream_t)s>>>(n, m, r, ns, q, x,
                                                           idx);
  return cudaGetLastError();
}

// See include/reference_queries.h.
GSA_API int nn3(int b, int n, int m, const float* q, const float* x, float* d,
                int* idx, void* s) {
  if (b < 0 || n < 0 || m < 0) return -2;
  if (!b || !n) return 0;
  if (!q || !d || !idx || (m && !x)) return -2;
  dim3 grid((n + kThreads - 1) / kThreads, b);
  count_launches();
  nn3_scan_kernel<<<grid, kThreads, 0, (cudaStream_t)s>>>(n, m, q, x, d, idx);
  return cudaGetLastError();
}
