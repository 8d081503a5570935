// SPDX-License-Identifier: Apache-2.0
#include "pool.cuh"

namespace gsa {
namespace {
cudaMemPool_t g_pool = nullptr;
int g_enabled = 1;

cudaError_t get_pool(cudaMemPool_t* out) {
  if (!g_pool) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e) return e;
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.handleTypes = cudaMemHandleTypeNone;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = device;
    e = cudaMemPoolCreate(&g_pool, &props);
    if (e) return e;
    uint64_t threshold = UINT64_MAX;
    e = cudaMemPoolSetAttribute(g_pool, cudaMemPoolAttrReleaseThreshold,
                                &threshold);
    if (e) return e;
  }
  *out = g_pool;
  return cudaSuccess;
}
}  // namespace

cudaError_t pool_alloc(void** p, size_t bytes, cudaStream_t s) {
  *p = nullptr;
  if (bytes == 0) bytes = 16;
  if (!g_enabled) return cudaMallocAsync(p, bytes, s);
  cudaMemPool_t pool;
  cudaError_t e = get_pool(&pool);
  if (e) return e;
  return cudaMallocFromPoolAsync(p, bytes, pool, s);
}

cudaError_t pool_free(void* p, cudaStream_t s) {
  if (!p) return cudaSuccess;
  return cudaFreeAsync(p, s);
}

void pool_set_enabled(int enabled) { g_enabled = enabled; }

cudaError_t pool_peaks(uint64_t* used, uint64_t* reserved) {
  if (!g_pool) {
    *used = 0;
    *reserved = 0;
    return cudaSuccess;
  }
  cudaError_t e =
      cudaMemPoolGetAttribute(g_pool, cudaMemPoolAttrUsedMemHigh, used);
  if (e) return e;
  return cudaMemPoolGetAttribute(g_pool, cudaMemPoolAttrReservedMemHigh,
                                 reserved);
}

cudaError_t pool_reset_peaks() {
  if (!g_pool) return cudaSuccess;
  uint64_t zero = 0;
  cudaError_t e =
      cudaMemPoolSetAttribute(g_pool, cudaMemPoolAttrUsedMemHigh, &zero);
  if (e) return e;
  return cudaMemPoolSetAttribute(g_pool, cudaMemPoolAttrReservedMemHigh, &zero);
}

}  // namespace gsa
