/* SPDX-License-Identifier: Apache-2.0
 *
 * reference_queries: original-order brute-force radius and 3NN scans for
 * B200 (sm_100a).  Shared library: gsa_b200/_native/reference_queries.so
 *
 * Drop-in for the C ABI of GSA's csrc/reference_queries.cu (the FlashFPS /
 * OpenPoints query kernels), as bound by gsa/reference.py:11-14.  Pointers
 * are DEVICE pointers; `s` is a cudaStream_t.  Returns 0 or a cudaError_t
 * value; -2 for a negative size, ns < 1 or a null buffer.  An empty batch
 * (b == 0, or no queries) is a no-op returning 0.
 */
#ifndef GSA_B200_REFERENCE_QUERIES_H
#define GSA_B200_REFERENCE_QUERIES_H

#ifdef __cplusplus
extern "C" {
#endif

/* Ordered ball query over b batch items: q (b, m, 3) queries, x (b, n, 3)
 * support, idx (b, m, ns) int32.  A row with at least one support point at
 * d2 < r*r receives the first ns such IDs in ascending order padded with the
 * first; a row without one is left untouched.
 * Replaces: int ball(int, int, int, float, int, const float*, const float*,
 *           int*, void*) -- GSA csrc/reference_queries.cu:112 */
int ball(int b, int n, int m, float r, int ns, const float* q, const float* x,
         int* idx, void* s);

/* Three nearest neighbours over b batch items: q (b, n, 3) queries ("unknown"),
 * x (b, m, 3) support ("known"), d (b, n, 3) float32 squared distances and
 * idx (b, n, 3) int32; finite distances only, (d2, id) order, missing
 * entries (inf, 0).
 * Replaces: int nn3(int, int, int, const float*, const float*, float*, int*,
 *           void*) -- GSA csrc/reference_queries.cu:118 */
int nn3(int b, int n, int m, const float* q, const float* x, float* d,
        int* idx, void* s);

/* Extension (no counterpart in the reference): total kernel launches this
 * library has issued since it was loaded. */
int launch_counter(unsigned long long* total);

#ifdef __cplusplus
}
#endif

#endif
