// SPDX-License-Identifier: Apache-2.0
// Reuse-cache lookup that allocates nothing.
//
// The session's reuse check runs in two steps: compare the current support
// and query prefix with each candidate's snapshots (coords_mismatch writes
// one flag per comparison into a caller-provided device buffer), then copy
// the rows of the first candidate whose two flags are clear (reuse_rows).
// That flag buffer is scratch memory the caller has to allocate.
//
// Some callers cannot allocate device memory at the point of the lookup:
// code running under a framework's caching allocator that must not be
// bypassed with cudaMalloc, latency-critical loops where cudaMalloc/cudaFree
// would synchronise the device and stall other streams, and deployments
// whose device footprint is fixed after start-up.  reuse_lookup_static
// performs the same lookup with its flags in a fixed file-scope device array
// (kStaticCandidates * 2 ints, 512 bytes), which every GPU that loads this
// library holds until the process exits.
//
// Set-up: a call outside stream capture, with the device current, looks up
// the array's device address with cudaGetSymbolAddress (host code cannot use
// the array's name as a device pointer) and caches it for that device; a
// call during capture uses that cached address, so make one call on each
// device before any stream capture.  All calls share the array and it
// keeps the previous call's contents, so every call clears its flags first;
// calls whose work overlaps on the GPU (different streams, no ordering)
// race on the array.  No call allocates or frees memory.
#include <mutex>
#include "common.cuh"

namespace gsa {
namespace {

constexpr int kStaticCandidates = 64;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int g_lookup_flags[2 * kStaticCandidates];

std::mutex g_setup_mutex;
int* g_flag_ptr[kMaxDevices] = {};

// Device address of g_lookup_flags on the current device.  Outside stream
// capture the address is looked up on every call (cudaGetSymbolAddress
// allocates nothing), so a context re-created after cudaDeviceReset gets the
// array's new address; during capture the address cached by the last call
// outside capture on this device is used (none cached: an error).
cudaError_t flags_on_current_device(cudaStream_t s, int** out) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e) return e;
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(s, &capture);
  if (e) return e;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (capture == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_lookup_flags);
    if (e) return e;
    g_flag_ptr[device] = static_cast<int*>(p);
  } else if (!g_flag_ptr[device]) {
    return cudaErrorStreamCaptureUnsupported;
  }
  *out = g_flag_ptr[device];
  return cudaSuccess;
}

struct LookupArgs {
  const float* cur[2];  // current support, current query prefix
  long long n[2];       // floats compared for support / query
  const float* saved[2][kStaticCandidates];
  const int* cached[kStaticCandidates];
  int count;
};

// Pair p: candidate p / 2, support (p even) or query prefix (p odd).  16-byte
// loads when both arrays are 16-byte aligned.
__global__ void __launch_bounds__(256)
    lookup_compare_kernel(LookupArgs a, int* flags) {
  int p = blockIdx.y;
  int side = p & 1;
  const float* u = a.cur[side];
  const float* v = a.saved[side][p >> 1];
  long long n = a.n[side];
  bool diff = false;
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long tail = 0;
  if (((((uintptr_t)u) | ((uintptr_t)v)) & 15) == 0) {
    const float4* u4 = reinterpret_cast<const float4*>(u);
    const float4* v4 = reinterpret_cast<const float4*>(v);
    const long long n4 = n >> 2;
    for (long long i = t; i < n4; i += stride) {
      const float4 x = __ldcs(u4 + i), y = __ldcs(v4 + i);
      diff |= (x.x != y.x) | (x.y != y.y) | (x.z != y.z) | (x.w != y.w);
    }
    tail = n4 << 2;
  }
  for (long long i = tail + t; i < n; i += stride) diff |= u[i] != v[i];
  if (__any_sync(kFull, diff) && (threadIdx.x & 31) == 0) flags[p] = 1;
}

__global__ void __launch_bounds__(256)
    lookup_gather_kernel(LookupArgs a, const int* flags, int src_ld, int rows,
                         int cols, int* dst, int* hit) {
  int c = 0;
  while (c < a.count && (flags[2 * c] | flags[2 * c + 1])) ++c;
  if (blockIdx.x == 0 && threadIdx.x == 0 && hit) *hit = c < a.count ? c : -1;
  if (c >= a.count) return;
  const int* src = a.cached[c];
  long long total = (long long)rows * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
       i < total; i += (long long)gridDim.x * blockDim.x) {
    long long row = i / cols, col = i - row * cols;
    dst[i] = src[row * src_ld + col];
  }
}

unsigned blocks_for_work(long long work) {
  long long b = (work + 255) / 256;
  return (unsigned)(b < 1 ? 1 : (b > 1184 ? 1184 : b));
}

}  // namespace
}  // namespace gsa

using namespace gsa;

// See include/gsa_bvh.h.
GSA_API int reuse_lookup_static(int count, const float* x, long long nx,
                                const float* q, long long nq,
                                const float* const* saved_x,
                                const float* const* saved_q,
                                const int* const* cached, int src_ld,
                                int rows, int cols, int* dst, int* hit,
                                void* stream) {
  if (count > kStaticCandidates) return -4;  // beyond the fixed flag array
  if (count < 1 || nx < 0 || nq < 0 || rows < 0 || cols < 1 || src_ld < cols)
    return -2;
  if (!x || !q || !saved_x || !saved_q || !cached || (rows && !dst)) return -2;
  cudaStream_t s = (cudaStream_t)stream;
  int* flags = nullptr;
  cudaError_t e = flags_on_current_device(s, &flags);
  if (e) return e;
  LookupArgs a = {};
  a.cur[0] = x;
  a.cur[1] = q;
  a.n[0] = nx;
  a.n[1] = nq;
  a.count = count;
  for (int c = 0; c < count; ++c) {
    if (!saved_x[c] || !saved_q[c] || !cached[c]) return -2;
    a.saved[0][c] = saved_x[c];
    a.saved[1][c] = saved_q[c];
    a.cached[c] = cached[c];
  }
  e = cudaMemsetAsync(flags, 0, sizeof(int) * 2 * count, s);
  if (e) return e;
  dim3 grid(blocks_for_work(nx > nq ? nx : nq), 2 * count);
  count_launches(2);
  lookup_compare_kernel<<<grid, 256, 0, s>>>(a, flags);
  lookup_gather_kernel<<<blocks_for_work((long long)rows * cols), 256, 0, s>>>(
      a, flags, src_ld, rows, cols, dst, hit);
  return cudaGetLastError();
}
