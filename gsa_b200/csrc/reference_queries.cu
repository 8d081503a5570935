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
// B200 execution: one warp per query.  Lane l tests support IDs l, l+32, ...
// in ascending blocks of 32; for the radius scan a ballot orders each block's
// hits by ID, so the row is written in scan order and the warp stops once it
// holds `ns` hits.  For 3NN each lane keeps the best three of its IDs and the
// warp merges them by shuffles in (d2, id) order, which is the order an
// ascending scan with strict `<` produces.  One warp per query keeps a call
// with few queries (the small supports the session sends here) spread over
// the SMs instead of a few threads each scanning the whole support.
#include <algorithm>
#include "common.cuh"

namespace gsa {
namespace {

constexpr int kWarps = 8;  // queries per block

__global__ void __launch_bounds__(kWarps * 32)
    ball_scan_kernel(int n, int m, float radius, int ns, const float* q,
                     const float* x, int* idx) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= m) return;  // warp-uniform
  const long long row = (long long)m * blockIdx.y + t;
  const float* qp = q + 3ll * row;
  const float* xb = x + 3ll * n * blockIdx.y;
  int* o = idx + row * ns;
  const float px = qp[0], py = qp[1], pz = qp[2];
  const float r2 = __fmul_rn(radius, radius);
  const unsigned lt = (1u << lane) - 1u;
  int cnt = 0, first = 0;
  for (int base = 0; base < n && cnt < ns; base += 32) {
    const int k = base + lane;
    bool hit = false;
    if (k < n) {
      const float* p = xb + 3ll * k;
      hit = exact_d2(px, py, pz, p[0], p[1], p[2]) < r2;
    }
    const unsigned hm = __ballot_sync(kFull, hit);
    if (!hm) continue;  // warp-uniform
    if (!cnt) first = base + __ffs(hm) - 1;
    const int slot = cnt + __popc(hm & lt);
    if (hit && slot < ns) o[slot] = k;
    cnt += __popc(hm);
  }
  // pad with the first hit; a row without one stays untouched
  if (cnt)
    for (int s = cnt + lane; s < ns; s += 32) o[s] = first;
}

// (d, i) before (e, j) in (squared distance, ID) order.
__device__ __forceinline__ bool before(float d, int i, float e, int j) {
  return d < e || (d == e && i < j);
}

__global__ void __launch_bounds__(kWarps * 32)
    nn3_scan_kernel(int n, int m, const float* q, const float* x, float* d,
                    int* idx) {
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= n) return;  // warp-uniform
  const long long row = (long long)n * blockIdx.y + t;
  const float* qp = q + 3ll * row;
  const float* xb = x + 3ll * m * blockIdx.y;
  const float px = qp[0], py = qp[1], pz = qp[2];
  const float inf = __int_as_float(0x7f800000);
  float b0 = inf, b1 = inf, b2 = inf;
  int i0 = INT_MAX, i1 = INT_MAX, i2 = INT_MAX;
  for (int k = lane; k < m; k += 32) {
    const float* p = xb + 3ll * k;
    const float v = exact_d2(px, py, pz, p[0], p[1], p[2]);
    if (v < b2) {  // false for +inf and NaN; ascending k keeps lower IDs
      if (v < b1) {
        b2 = b1;
        i2 = i1;
        if (v < b0) {
          b1 = b0;
          i1 = i0;
          b0 = v;
          i0 = k;
        } else {
          b1 = v;
          i1 = k;
        }
      } else {
        b2 = v;
        i2 = k;
      }
    }
  }
  // butterfly merge of two (d2, id)-sorted triples; every lane ends with the
  // warp's best three
  for (int off = 16; off; off >>= 1) {
    const float e0 = __shfl_xor_sync(kFull, b0, off);
    const float e1 = __shfl_xor_sync(kFull, b1, off);
    const float e2 = __shfl_xor_sync(kFull, b2, off);
    const int j0 = __shfl_xor_sync(kFull, i0, off);
    const int j1 = __shfl_xor_sync(kFull, i1, off);
    const int j2 = __shfl_xor_sync(kFull, i2, off);
    bool a = before(b0, i0, e0, j0);
    const float r0 = a ? b0 : e0;
    const int s0 = a ? i0 : j0;
    // heads left after the first pick: (x0, x1) of one list, (y0, y1) of the
    // other
    const float x0 = a ? b1 : b0, x1 = a ? b2 : b1;
    const int u0 = a ? i1 : i0, u1 = a ? i2 : i1;
    const float y0 = a ? e0 : e1, y1 = a ? e1 : e2;
    const int w0 = a ? j0 : j1, w1 = a ? j1 : j2;
    a = before(x0, u0, y0, w0);
    const float r1 = a ? x0 : y0;
    const int s1 = a ? u0 : w0;
    const float z = a ? x1 : x0, y = a ? y0 : y1;
    const int uz = a ? u1 : u0, wy = a ? w0 : w1;
    const bool c = before(z, uz, y, wy);
    b0 = r0;
    i0 = s0;
    b1 = r1;
    i1 = s1;
    b2 = c ? z : y;
    i2 = c ? uz : wy;
  }
  if (lane < 3) {
    const float v = lane == 0 ? b0 : (lane == 1 ? b1 : b2);
    const int id = lane == 0 ? i0 : (lane == 1 ? i1 : i2);
    d[3 * row + lane] = v;
    idx[3 * row + lane] = id == INT_MAX ? 0 : id;
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
  dim3 grid((m + kWarps - 1) / kWarps, b);
  count_launches();
  ball_scan_kernel<<<grid, kWarps * 32, 0, (cudaStream_t)s>>>(n, m, r, ns, q,
                                                             x, idx);
  return cudaGetLastError();
}

// See include/reference_queries.h.
GSA_API int nn3(int b, int n, int m, const float* q, const float* x, float* d,
                int* idx, void* s) {
  if (b < 0 || n < 0 || m < 0) return -2;
  if (!b || !n) return 0;
  if (!q || !d || !idx || (m && !x)) return -2;
  dim3 grid((n + kWarps - 1) / kWarps, b);
  count_launches();
  nn3_scan_kernel<<<grid, kWarps * 32, 0, (cudaStream_t)s>>>(n, m, q, x, d,
                                                            idx);
  return cudaGetLastError();
}
