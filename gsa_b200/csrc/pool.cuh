// SPDX-License-Identifier: Apache-2.0
// Stream-ordered device allocations for trees and build scratch.  Mirrors the
// behaviour of the GSA native allocator (csrc/gsa_bvh.cu:13-44): a private
// cudaMemPool bound to the first device used, release threshold UINT64_MAX,
// switchable to the device's default pool with set_pool_mode(0).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace gsa {

cudaError_t pool_alloc(void** p, size_t bytes, cudaStream_t s);
cudaError_t pool_free(void* p, cudaStream_t s);
void pool_set_enabled(int enabled);
cudaError_t pool_peaks(uint64_t* used, uint64_t* reserved);
cudaError_t pool_reset_peaks();

}  // namespace gsa
