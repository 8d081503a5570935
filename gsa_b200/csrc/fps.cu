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
#include <algorithm>
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

// The first m points of the order of each scene (m <= n); start[b] null
// starts every scene at index 0.
__global__ void __launch_bounds__(kFpsThreads)
    fps_kernel(int n, int m, const float* x, const int* start, int* order) {
  extern __shared__ float mind[];
  __shared__ float wv[32];
  __shared__ int wi[32];
  __shared__ int cur_s;
  int b = blockIdx.x;
  const float* xb = x + 3ll * n * b;
  int* ob = order + (long long)m * b;
  for (int i = threadIdx.x; i < n; i += kFpsThreads)
    mind[i] = __int_as_float(0x7f800000);
  if (threadIdx.x == 0) cur_s = start ? start[b] : 0;
  __syncthreads();
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int it = 0; it < m; ++it) {
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

// ---------------------------------------------------------------------------
// Large scenes: one cooperative grid (every block resident) per scene, PER
// points per thread in registers.  Per step each block reduces its best
// (distance, lowest index), one atomicMax on a packed 64-bit key per block
// selects the global best, and a grid barrier separates steps.  The winner
// slot is triple-buffered so it can be cleared two steps ahead without a
// second barrier.
#ifndef GSA_FPS_BARRIER_SPINS
#define GSA_FPS_BARRIER_SPINS (1ll << 24)
#endif
constexpr long long kBarrierSpins = GSA_FPS_BARRIER_SPINS;
// Test builds only: the block with this index leaves the kernel at its first
// barrier without arriving, so every other block's bounded wait runs out and
// the call reports the error flag (-1: none).
#ifndef GSA_FPS_DROP_BLOCK
#define GSA_FPS_DROP_BLOCK -1
#endif

__device__ __forceinline__ unsigned order_key(float f) {
  unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Grid barrier with a bounded wait: on timeout it sets *err and returns.
__device__ void grid_barrier(unsigned* count, unsigned* gen, int* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned g = *reinterpret_cast<volatile unsigned*>(gen);
    __threadfence();
    if (atomicAdd(count, 1u) == gridDim.x - 1) {
      *count = 0;
      __threadfence();
      atomicAdd(gen, 1u);
    } else {
      long long spins = 0;
      while (*reinterpret_cast<volatile unsigned*>(gen) == g) {
        if (++spins > kBarrierSpins) {
          atomicExch(err, 1);
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
  }
  __syncthreads();
}

template <int PER>
__global__ void __launch_bounds__(kFpsThreads)
    fps_grid_kernel(int n, int m, const float* x, int start, int* order,
                    unsigned long long* best, unsigned* bar, int* err) {
  __shared__ unsigned long long wbest[32];
  const int threads = gridDim.x * kFpsThreads;
  const int tid = blockIdx.x * kFpsThreads + threadIdx.x;
  float px[PER], py[PER], pz[PER], md[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    int i = tid + k * threads;
    md[k] = i < n ? __int_as_float(0x7f800000) : -2.f;
    px[k] = i < n ? x[3ll * i] : 0.f;
    py[k] = i < n ? x[3ll * i + 1] : 0.f;
    pz[k] = i < n ? x[3ll * i + 2] : 0.f;
  }
  int cur = start;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int it = 0; it < m; ++it) {
    if (tid == 0) order[it] = cur;
    float cx = __ldg(x + 3ll * cur), cy = __ldg(x + 3ll * cur + 1),
          cz = __ldg(x + 3ll * cur + 2);
    unsigned long long mine = 0;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      int i = tid + k * threads;
      if (i == cur) {
        md[k] = -1.f;
      } else if (md[k] >= 0.f) {
        md[k] = fminf(md[k], exact_d2(px[k], py[k], pz[k], cx, cy, cz));
      }
      if (i < n) {
        unsigned long long key =
            ((unsigned long long)order_key(md[k]) << 32) | (0xffffffffu - (unsigned)i);
        mine = key > mine ? key : mine;
      }
    }
    for (int o = 16; o; o >>= 1) {
      unsigned long long u = __shfl_xor_sync(kFull, mine, o);
      mine = u > mine ? u : mine;
    }
    if (lane == 0) wbest[warp] = mine;
    __syncthreads();
    if (warp == 0) {
      mine = lane < kFpsThreads / 32 ? wbest[lane] : 0;
      for (int o = 16; o; o >>= 1) {
        unsigned long long u = __shfl_xor_sync(kFull, mine, o);
        mine = u > mine ? u : mine;
      }
      if (lane == 0) atomicMax(best + it % 3, mine);
    }
    if (GSA_FPS_DROP_BLOCK >= 0 && (int)blockIdx.x == GSA_FPS_DROP_BLOCK) return;
    grid_barrier(bar, bar + 1, err);
    if (*reinterpret_cast<volatile int*>(err)) return;
    unsigned long long win = *reinterpret_cast<volatile unsigned long long*>(best + it % 3);
    cur = (int)(0xffffffffu - (unsigned)(win & 0xffffffffu));
    if (tid == 0) best[(it + 2) % 3] = 0;
  }
}

template <int PER>
cudaError_t launch_fps_grid(int n, int m, const float* x, int start,
                            int* order, unsigned long long* best,
                            unsigned* bar, int* err, int blocks,
                            cudaStream_t s) {
  void* args[] = {&n, &m, &x, &start, &order, &best, &bar, &err};
  return cudaLaunchCooperativeKernel((const void*)fps_grid_kernel<PER>,
                                     dim3(blocks), dim3(kFpsThreads), args, 0,
                                     s);
}

}  // namespace
}  // namespace gsa

using namespace gsa;

namespace {

constexpr size_t kFpsSmemMax = 200 * 1024;  // running minima in shared memory

cudaError_t fps_large(int n, int m, const float* x, int start, int* order,
                      void* scratch, int* err, cudaStream_t s, int* code) {
  *code = 0;
  int device = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (!e) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (!e)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, fps_grid_kernel<8>, kFpsThreads, 0);
  if (e) return e;
  int blocks = sms * std::min(per_sm, 1);
  long long threads = (long long)blocks * kFpsThreads;
  if (n > threads * 8) {  // at most 8 points per thread
    *code = -2;
    return cudaSuccess;
  }
  unsigned long long* best = static_cast<unsigned long long*>(scratch);
  unsigned* bar = reinterpret_cast<unsigned*>(best + 3);
  e = cudaMemsetAsync(scratch, 0, 64, s);
  if (!e) e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e) return e;
  count_launches();
  if (n <= threads * 2)
    e = launch_fps_grid<2>(n, m, x, start, order, best, bar, err, blocks, s);
  else
    e = launch_fps_grid<8>(n, m, x, start, order, best, bar, err, blocks, s);
  return e ? e : cudaGetLastError();
}

cudaError_t fps_small(int b, int n, int m, const float* x, const int* start,
                      int* order, cudaStream_t s) {
  size_t smem = sizeof(float) * (size_t)n;
  cudaError_t e = cudaFuncSetAttribute(
      fps_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e) return e;
  count_launches();
  fps_kernel<<<b, kFpsThreads, smem, s>>>(n, m, x, start, order);
  return cudaGetLastError();
}

}  // namespace

// See include/gsa_bvh.h.
GSA_API int fps_order_large(int n, const float* x, int start, int* order,
                            void* scratch, int* err, void* stream) {
  if (n < 1 || !x || !order || !scratch || !err || start < 0 || start >= n)
    return -2;
  int code = 0;
  cudaError_t e = fps_large(n, n, x, start, order, scratch, err,
                            (cudaStream_t)stream, &code);
  return e ? (int)e : code;
}

// See include/gsa_bvh.h.
GSA_API int fps_order(int b, int n, const float* x, const int* start,
                      int* order, void* stream) {
  if (b < 0 || n < 0) return -2;
  if (!b || !n) return 0;
  if (sizeof(float) * (size_t)n > kFpsSmemMax) return -2;
  if (!x || !start || !order) return -2;
  return (int)fps_small(b, n, n, x, start, order, (cudaStream_t)stream);
}

// See include/gsa_bvh.h.
GSA_API int furthest_point_sample(int b, int n, int m, const float* x,
                                  float* temp, int* idx, void* stream) {
  if (b < 0 || n < 0 || m < 0 || m > n) return -2;
  if (!b || !m) return 0;
  if (!x || !idx) return -2;
  cudaStream_t s = (cudaStream_t)stream;
  if (sizeof(float) * (size_t)n <= kFpsSmemMax)
    return (int)fps_small(b, n, m, x, nullptr, idx, s);
  // one scene per cooperative grid; temp (b*n floats) holds its barrier
  // words and the error flag
  if (!temp) return -2;
  for (int i = 0; i < b; ++i) {
    float* t = temp + (long long)n * i;
    int code = 0;
    cudaError_t e = fps_large(n, m, x + 3ll * n * i, 0, idx + (long long)m * i,
                              t, reinterpret_cast<int*>(t + 16), s, &code);
    if (e) return (int)e;
    if (code) return code;
  }
  return 0;
}
