// SPDX-License-Identifier: Apache-2.0
// QuerySession result-row reuse on the device.
//
// GSA admits a cached radius row (gsa/session.py:104-114) when the support and
// the query prefix equal the retained snapshots, tested with one torch.equal
// (a kernel plus a host synchronisation) per comparison, then copies
// cached[:Q, :k].  Here every candidate comparison of a call runs in ONE
// launch (coords_mismatch), the first candidate whose support and query both
// match is selected and its rows gathered on the device (reuse_rows), and the
// host reads the flags once to keep the session statistics exact.
//
// Equality is IEEE value equality of float32 elements, the semantics of
// torch.equal: NaN never equals, -0 equals +0.
#include <algorithm>
#include "common.cuh"

namespace gsa {
namespace {

constexpr int kMaxPairs = 64;

struct PairChunk {
  const float* a[kMaxPairs];
  const float* b[kMaxPairs];
  long long n[kMaxPairs];
};

__global__ void __launch_bounds__(256)
    mismatch_kernel(PairChunk c, int* flags) {
  int p = blockIdx.y;
  const float* a = c.a[p];
  const float* b = c.b[p];
  long long n = c.n[p];
  bool diff = false;
  long long stride = (long long)gridDim.x * blockDim.x;
  long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  bool vec = ((((uintptr_t)a) | ((uintptr_t)b)) & 15) == 0;
  if (vec) {
    long long n4 = n >> 2;
    const float4* a4 = reinterpret_cast<const float4*>(a);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    for (long long i = t; i < n4; i += stride) {
      float4 u = __ldcs(a4 + i), v = __ldcs(b4 + i);
      diff |= (u.x != v.x) | (u.y != v.y) | (u.z != v.z) | (u.w != v.w);
    }
    for (long long i = (n4 << 2) + t; i < n; i += stride) diff |= a[i] != b[i];
  } else {
    for (long long i = t; i < n; i += stride) diff |= a[i] != b[i];
  }
  if (__any_sync(kFull, diff) && (threadIdx.x & 31) == 0) flags[p] = 1;
}

struct RowChunk {
  const int* src[kMaxPairs];
};

// dst[i, j] = src[i * src_ld + j] for i < rows, j < cols (grid-stride).
__device__ void copy_rows(const int* src, int src_ld, int rows, int cols,
                          int* dst) {
  long long total = (long long)rows * cols;
  long long stride = (long long)gridDim.x * blockDim.x;
  if (cols == src_ld && ((((uintptr_t)src) | ((uintptr_t)dst)) & 15) == 0 &&
      (total & 3) == 0) {
    const int4* s4 = reinterpret_cast<const int4*>(src);
    int4* d4 = reinterpret_cast<int4*>(dst);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
         i < (total >> 2); i += stride)
      d4[i] = __ldcs(s4 + i);
    return;
  }
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
       i < total; i += stride) {
    long long row = i / cols, col = i - row * cols;
    dst[i] = src[row * src_ld + col];
  }
}

// Copies the rows of the first candidate c with flags[2c] == flags[2c+1] == 0
// (support and query prefix both equal); records c, or -1, in *hit.
__global__ void __launch_bounds__(256)
    reuse_rows_kernel(RowChunk r, int count, const int* flags, int src_ld,
                      int rows, int cols, int* dst, int* hit) {
  int c = 0;
  while (c < count && (flags[2 * c] | flags[2 * c + 1])) ++c;
  if (blockIdx.x == 0 && threadIdx.x == 0 && hit) *hit = c < count ? c : -1;
  if (c >= count) return;
  copy_rows(r.src[c], src_ld, rows, cols, dst);
}

__global__ void __launch_bounds__(256)
    gather_rows_kernel(const int* src, int src_ld, int rows, int cols,
                       int* dst) {
  copy_rows(src, src_ld, rows, cols, dst);
}

// Pair p = (a + p*a_stride, b + p*b_stride), nfloat values each.
__global__ void __launch_bounds__(256)
    mismatch_strided_kernel(const float* a, long long a_stride, const float* b,
                            long long b_stride, long long n, int* flags,
                            int flag_stride) {
  long long p = blockIdx.y;
  const float* u = a + p * a_stride;
  const float* v = b + p * b_stride;
  bool diff = false;
  long long stride = (long long)gridDim.x * blockDim.x;
  long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (((((uintptr_t)u) | ((uintptr_t)v)) & 15) == 0) {
    const float4* u4 = reinterpret_cast<const float4*>(u);
    const float4* v4 = reinterpret_cast<const float4*>(v);
    long long n4 = n >> 2;
    for (long long i = t; i < n4; i += stride) {
      float4 x = __ldcs(u4 + i), y = __ldcs(v4 + i);
      diff |= (x.x != y.x) | (x.y != y.y) | (x.z != y.z) | (x.w != y.w);
    }
    for (long long i = (n4 << 2) + t; i < n; i += stride) diff |= u[i] != v[i];
  } else {
    for (long long i = t; i < n; i += stride) diff |= u[i] != v[i];
  }
  if (__any_sync(kFull, diff) && (threadIdx.x & 31) == 0)
    flags[p * flag_stride] = 1;
}

// Scene i copies its rows unless its support or query flag is set.
__global__ void __launch_bounds__(256)
    reuse_rows_batch_kernel(const int* src, long long src_stride, int src_ld,
                            const int* flags, int rows, int cols, int* dst,
                            long long dst_stride, int* hits) {
  long long i = blockIdx.y;
  bool hit = !flags || !(flags[2 * i] | flags[2 * i + 1]);
  if (hits && blockIdx.x == 0 && threadIdx.x == 0) hits[i] = hit;
  if (hit)
    copy_rows(src + i * src_stride, src_ld, rows, cols, dst + i * dst_stride);
}

inline unsigned copy_blocks(long long work) {
  long long b = (work + 255) / 256;
  return (unsigned)std::max<long long>(1, std::min<long long>(b, 148 * 8));
}

}  // namespace
}  // namespace gsa

using namespace gsa;

// See include/gsa_bvh.h.
GSA_API int coords_mismatch(int count, const float* const* a,
                            const float* const* b, const long long* nfloat,
                            int* flags, void* stream) {
  if (count < 0 || (count && (!a || !b || !nfloat || !flags))) return -2;
  if (!count) return 0;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(int) * count, s);
  if (e) return e;
  for (int c0 = 0; c0 < count; c0 += kMaxPairs) {
    PairChunk c;
    int k = std::min(kMaxPairs, count - c0);
    long long longest = 0;
    for (int i = 0; i < kMaxPairs; ++i) {
      bool on = i < k;
      c.a[i] = on ? a[c0 + i] : nullptr;
      c.b[i] = on ? b[c0 + i] : nullptr;
      c.n[i] = on ? nfloat[c0 + i] : 0;
      if (on && c.n[i] < 0) return -2;
      if (on) longest = std::max(longest, c.n[i]);
    }
    dim3 grid(copy_blocks((longest + 3) / 4), k);
    count_launches();
    mismatch_kernel<<<grid, 256, 0, s>>>(c, flags + c0);
  }
  return cudaGetLastError();
}

// See include/gsa_bvh.h.
GSA_API int reuse_rows(int count, const int* const* cached, const int* flags,
                       int src_ld, int rows, int cols, int* dst, int* hit,
                       void* stream) {
  if (count < 1 || count > kMaxPairs || !cached || !flags || rows < 0 ||
      cols < 1 || src_ld < cols || (rows && !dst))
    return -2;
  RowChunk r;
  for (int i = 0; i < kMaxPairs; ++i) r.src[i] = i < count ? cached[i] : nullptr;
  cudaStream_t s = (cudaStream_t)stream;
  count_launches();
  reuse_rows_kernel<<<copy_blocks(((long long)rows * cols + 3) / 4), 256, 0,
                      s>>>(r, count, flags, src_ld, rows, cols, dst, hit);
  return cudaGetLastError();
}

// See include/gsa_bvh.h.
GSA_API int gather_rows(const int* src, int src_ld, int rows, int cols,
                        int* dst, void* stream) {
  if (rows < 0 || cols < 1 || src_ld < cols || (rows && (!src || !dst)))
    return -2;
  if (!rows) return 0;
  cudaStream_t s = (cudaStream_t)stream;
  count_launches();
  gather_rows_kernel<<<copy_blocks(((long long)rows * cols + 3) / 4), 256, 0,
                       s>>>(src, src_ld, rows, cols, dst);
  return cudaGetLastError();
}

// See include/gsa_bvh.h.
GSA_API int coords_mismatch_strided(int count, const float* a,
                                    long long a_stride, const float* b,
                                    long long b_stride, long long nfloat,
                                    int* flags, int flag_stride,
                                    void* stream) {
  if (count < 0 || nfloat < 0 || flag_stride < 1 || count > 65535) return -2;
  if (!count) return 0;
  if (!a || !b || !flags) return -2;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemset2DAsync(flags, sizeof(int) * flag_stride, 0,
                                    sizeof(int), count, s);
  if (e) return e;
  if (!nfloat) return 0;
  dim3 grid(copy_blocks((nfloat + 3) / 4), count);
  count_launches();
  mismatch_strided_kernel<<<grid, 256, 0, s>>>(a, a_stride, b, b_stride, nfloat,
                                               flags, flag_stride);
  return cudaGetLastError();
}

// See include/gsa_bvh.h.
GSA_API int reuse_rows_batch(int count, const int* src, long long src_stride,
                             int src_ld, const int* flags, int rows, int cols,
                             int* dst, long long dst_stride, int* hits,
                             void* stream) {
  if (count < 0 || count > 65535 || rows < 0 || cols < 1 || src_ld < cols)
    return -2;
  if (!count) return 0;
  if (!src || !dst) return -2;
  dim3 grid(copy_blocks(((long long)rows * cols + 3) / 4), count);
  count_launches();
  reuse_rows_batch_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
      src, src_stride, src_ld, flags, rows, cols, dst, dst_stride, hits);
  return cudaGetLastError();
}

// See include/gsa_bvh.h.
GSA_API int session_lookup(int count, const float* const* a,
                           const float* const* b, const long long* nfloat,
                           int nmemo, const int* const* cached, int src_ld,
                           int rows, int cols, int* dst, int* flags,
                           int* flags_host, void* stream) {
  if (count < 1 || nmemo < 0 || 2 * nmemo > count || nmemo > kMaxPairs ||
      !flags || !flags_host)
    return -2;
  int code = coords_mismatch(count, a, b, nfloat, flags, stream);
  if (code) return code;
  if (nmemo) {
    code = reuse_rows(nmemo, cached, flags, src_ld, rows, cols, dst, nullptr,
                      stream);
    if (code) return code;
  }
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemcpyAsync(flags_host, flags, sizeof(int) * count,
                                  cudaMemcpyDeviceToHost, s);
  if (!e) e = cudaStreamSynchronize(s);
  return (int)e;
}
