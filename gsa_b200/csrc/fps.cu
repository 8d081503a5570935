// SPDX-License-Identifier: Apache-2.0
// Farthest-point ordering of whole scenes, used to produce the FPS-ordered
// supports of the hierarchical workloads (prefixes n, n/4, n/16, ... of an FPS
// order are the sampled levels).  Deterministic and exact: the running
// minimum squared distance uses the engine's exact FP32 distance, already
// chosen points are marked -1, and ties pick the lowest index, so the order
// equals a sequential CPU implementation with the same rules.
//
// One 1024-thread block per scene; the running minimum lives in shared memory
// (4 bytes per point), coordinates are re-read from L2 each step.
#include "common.cuh"

namespace gsa {
namespace {

constexpr int kFpsThreads = 1024;

__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

__global__ void __launch_bounds__(kFpsThreads)
    fps_kernel(int n, const float* x, const int* start, int* order) {
  extern __shared__ float mind[];
  __shared__ float wv[32];
  __shared__ int wi[32];
  __shared__ int cur_s;
  int b = blockIdx.x;
  const float* xb = x + 3ll * n * b;
  int* ob = order + (long long)n * b;
  for (int i = threadIdx.x; i < n; i += kFpsThreads)
    mind[i] = __int_as_float(0x7f800000);
  if (threadIdx.x == 0) cur_s = start[b];
  __syncthreads();
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int it = 0; it < n; ++it) {
    int cur = cur_s;
    if (threadIdx.x == 0) ob[it] = cur;
    float cx = __ldg(xb + 3ll * cur), cy = __ldg(xb + 3ll * cur + 1),
          cz = __ldg(xb + 3ll * cur + 2);
    float bv = -2.f;
    int bi = INT_MAX;
    for (int i = threadIdx.x; i < n; i += kFpsThreads) {
      float v = mind[i];
      if (i == cur) {
        v = -1.f;
      } else if (v >= 0.f) {
        float d = exact_d2(__ldg(xb + 3ll * i), __ldg(xb + 3ll * i + 1),
                           __ldg(xb + 3ll * i + 2), cx, cy, cz);
        v = fminf(v, d);
      }
      mind[i] = v;
      better(bv, bi, v, i);
    }
    for (int o = 16; o; o >>= 1) {
      float v2 = __shfl_xor_sync(kFull, bv, o);
      int i2 = __shfl_xor_sync(kFull, bi, o);
      better(bv, bi, v2, i2);
    }
    if (lane == 0) {
      wv[warp] = bv;
      wi[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
      bv = wv[lane];
      bi = wi[lane];
      for (int o = 16; o; o >>= 1) {
        float v2 = __shfl_xor_sync(kFull, bv, o);
        int i2 = __shfl_xor_sync(kFull, bi, o);
        better(bv, bi, v2, i2);
      }
      if (lane == 0) cur_s = bi;
    }
    __syncthreads();
  }
}

}  // namespace
}  // namespace gsa

using namespace gsa;

// See include/gsa_bvh.h.
GSA_API int fps_order(int b, int n, const float* x, const int* start,
                      int* order, void* stream) {
  if (b < 0 || n < 0) return -2;
  if (!b || !n) return 0;
  size_t smem = sizeof(float) * (size_t)n;
  if (smem > 200 * 1024) return -2;
  if (!x || !start || !order) return -2;
  cudaError_t e = cudaFuncSetAttribute(
      fps_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e) return e;
  count_launches();
  fps_kernel<<<b, kFpsThreads, smem, (cudaStream_t)stream>>>(n, x, start,
                                                              order);
  return cudaGetLastError();
}
