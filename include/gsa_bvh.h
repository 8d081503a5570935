/* SPDX-License-Identifier: Apache-2.0
 *
 * gsa_bvh: exact prefix-BVH point queries for B200 (sm_100a).
 * Shared library: gsa_b200/_native/gsa_bvh.so
 *
 * Drop-in for the C ABI of GSA's csrc/gsa_bvh.cu (qmkkk/GSA), as bound by
 * gsa/runtime.py:13-26.  All pointers named x, q, d, ix, out, fallback, flags
 * and cached are DEVICE pointers on the current CUDA device; `stream` is a
 * cudaStream_t.  Every call is stream-ordered and does not synchronise the
 * host (except free_bvh with async_free == 0).
 *
 * Return codes (as in the reference): 0 success; a cudaError_t value for a
 * CUDA error; -1 build failure / invalid build argument; -2 invalid query
 * argument (bad m, level or ns); -3 invalid handle on free.
 *
 * Coordinates are contiguous float32 (N, 3).  Squared distance is
 * ((dx*dx + dy*dy) + dz*dz), round-to-nearest, no FMA, subnormals kept.
 */
#ifndef GSA_B200_GSA_BVH_H
#define GSA_B200_GSA_BVH_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Builds a tree over x[0..n).  prefix != 0 stores bounds for the four ordered
 * prefixes n, n/4, n/16, n/64 (levels 0..3) on one topology.  x is BORROWED:
 * it must stay alive and unchanged until free_bvh.  leaf >= 1 is the maximum
 * leaf size (clamped to 32; results never depend on it).
 * Replaces: int build_bvh(const float*, int, int, int, void**, void*)
 *           -- GSA csrc/gsa_bvh.cu:217 */
int build_bvh(const float* x, int n, int prefix, int leaf, void** out,
              void* stream);

/* Exact 3NN of nq queries against support IDs < m (3 <= m <= n).  level is
 * -1 (all-point bounds) or the prefix level whose size is >= m.  Writes
 * d[nq*3] ascending squared distances and ix[nq*3] IDs, ties by lower ID,
 * missing entries (inf, 0).  *fallback counts stack-overflow full scans.
 * Replaces: int query_bvh(void*, const float*, int, int, int, float*, int*,
 *           int*, void*) -- GSA csrc/gsa_bvh.cu:249 */
int query_bvh(void* h, const float* q, int nq, int m, int level, float* d,
              int* ix, int* fallback, void* stream);

/* Exact ordered radius query: per query the first ns (1..32) support IDs
 * < m (1 <= m <= n) with d2 < radius*radius, ascending, padded with the
 * first; a zero row when none qualifies.  out is int32 [nq*ns].
 * Replaces: int query_ball_bvh(void*, const float*, int, int, int, float,
 *           int, int*, int*, void*) -- GSA csrc/gsa_bvh.cu:344 */
int query_ball_bvh(void* h, const float* q, int nq, int m, int level,
                   float radius, int ns, int* out, int* fallback,
                   void* stream);

/* Releases a tree (stream-ordered); async_free == 0 also synchronises the
 * stream.  Replaces: int free_bvh(void*, int, void*)
 * -- GSA csrc/gsa_bvh.cu:258 */
int free_bvh(void* h, int async_free, void* stream);

/* 1: allocate from the library's private memory pool (default); 0: from the
 * device's default pool.  Replaces: int set_pool_mode(int)
 * -- GSA csrc/gsa_bvh.cu:356 */
int set_pool_mode(int enabled);

/* High-water marks of the private pool (0, 0 before first use).
 * Replaces: int pool_memory(uint64_t*, uint64_t*) -- GSA csrc/gsa_bvh.cu:360 */
int pool_memory(uint64_t* used_peak, uint64_t* reserved_peak);

/* Resets both high-water marks.
 * Replaces: int pool_reset_peak(void) -- GSA csrc/gsa_bvh.cu:373 */
int pool_reset_peak(void);

/* ---- Extensions without a counterpart in the reference ---------------- */

/* query_bvh / query_ball_bvh for query sets that are not the support's own
 * points (same arguments, same results).  The query kernels walk queries in
 * packets of neighbouring points, and query_bvh / query_ball_bvh take the
 * support's leaf order for them, which fits GSA's prefix queries (a query
 * array that is the support's first rows) exactly.  These take the queries'
 * own Morton order instead (one key sort of the nq points, scratch from the
 * library pool, freed stream-ordered), so shuffled or unrelated query sets
 * keep coherent packets; their 3NN rows take the per-query walk, the window
 * bound needing support points.  Same extension of GSA csrc/gsa_bvh.cu:249
 * and :344. */
int query_bvh_unordered(void* h, const float* q, int nq, int m, int level,
                        float* d, int* ix, int* fallback, void* stream);
int query_ball_bvh_unordered(void* h, const float* q, int nq, int m,
                             int level, float radius, int ns, int* out,
                             int* fallback, void* stream);

/* Forest of b independent trees (one per scene) over one concatenated point
 * array: tree i owns x[seg[i]..seg[i+1]) (seg is a HOST array of b+1
 * ascending offsets starting at 0, every tree non-empty).  All trees are
 * built by the same kernel launches.  Replaces the per-scene loop of
 * build_bvh calls (GSA csrc/gsa_bvh.cu:217) for batched inference. */
int build_bvh_batch(const float* x, const int* seg, int b, int prefix,
                    int leaf, void** out, void* stream);

/* Rebuilds a forest (from build_bvh_batch or build_bvh) in place from points
 * x laid out as at its creation (same scene sizes; x may be a new address,
 * and is borrowed like build_bvh's).  The first call on a forest allocates
 * the build temporaries from the library pool and keeps them until free_bvh;
 * every later call enqueues the build kernels only, so a rebuild followed by
 * queries can be captured in a CUDA graph and replayed for new coordinate
 * values.  Returns 0 or a cudaError_t; -1 for a null handle or x.  No
 * counterpart in the reference, which builds a new tree per call
 * (csrc/gsa_bvh.cu:217). */
int rebuild_bvh_batch(void* h, const float* x, void* stream);

/* Radius query on every tree of a forest in one launch.  Tree i answers
 * qseg[i+1]-qseg[i] queries read from rows q[qstart[i]..) (qstart null: from
 * row qseg[i]) and writes output rows qseg[i].. of out (ns ints per row).
 * qstart and qseg are device int arrays, qseg_host the host copy of qseg
 * (b+1 offsets from 0).  Tree i searches support IDs < m_i where m_i = m if
 * m > 0, else its level size n_i >> (2*level) (n_i for level -1); m_i must
 * not exceed that level size.  Passing q = the forest's own points and
 * qstart = seg answers each scene's own prefix without copying it. */
int query_ball_bvh_batch(void* h, const float* q, const int* qstart,
                         const int* qseg, const int* qseg_host, int m,
                         int level, float radius, int ns, int* out,
                         int* fallback, void* stream);

/* 3NN on every tree of a forest in one launch (same layout as above; every
 * tree with queries needs m_i >= 3). */
int query_bvh_batch(void* h, const float* q, const int* qstart,
                    const int* qseg, const int* qseg_host, int m, int level,
                    float* d, int* ix, int* fallback, void* stream);

/* Trees, points, stored levels and leaf size of a handle (any may be null). */
int bvh_info(void* h, int* trees, int* points, int* levels, int* leaf);

/* Reuse-cache check: for each pair c < count, flags[c] = 0 when the nfloat[c]
 * float32 values at a[c] and b[c] are all equal (IEEE ==, the semantics of
 * torch.equal: NaN never equal, -0 == +0), else 1.  a, b, nfloat are HOST
 * arrays of device pointers / counts; flags is device int[count].  One
 * launch for all pairs.  Replaces the per-comparison torch.equal of
 * GSA gsa/session.py:39-43. */
int coords_mismatch(int count, const float* const* a, const float* const* b,
                    const long long* nfloat, int* flags, void* stream);

/* Reuse-cache gather: selects the first candidate c < count (count <= 64)
 * whose flags[2c] and flags[2c+1] are both 0 and copies
 * cached[c][i*src_ld + j] to dst[i*cols + j] for i < rows, j < cols; writes c
 * (or -1 when none matches) to *hit (device int, may be null).  cached is a
 * HOST array of device pointers.  Replaces `out.copy_(cached[:len(q), :k])`
 * of GSA gsa/session.py:111. */
int reuse_rows(int count, const int* const* cached, const int* flags,
               int src_ld, int rows, int cols, int* dst, int* hit,
               void* stream);

/* dst[i*cols + j] = src[i*src_ld + j] for i < rows, j < cols.  Replaces
 * `out.copy_(result[:, :k])` of GSA gsa/session.py:128. */
int gather_rows(const int* src, int src_ld, int rows, int cols, int* dst,
                void* stream);

/* Batched reuse check over `count` scenes in one launch: flags[p*flag_stride]
 * = 0 when the nfloat values at a + p*a_stride and b + p*b_stride are all
 * equal (IEEE ==), else 1; the other flag slots are untouched.  Batched form
 * of the session's support/query snapshot comparisons (gsa/session.py:104-114)
 * for scenes laid out at a fixed stride. */
int coords_mismatch_strided(int count, const float* a, long long a_stride,
                            const float* b, long long b_stride,
                            long long nfloat, int* flags, int flag_stride,
                            void* stream);

/* Batched reuse gather: scene p < count copies
 * src[p*src_stride + i*src_ld + j] to dst[p*dst_stride + i*cols + j]
 * (i < rows, j < cols) when flags is null or flags[2p] == flags[2p+1] == 0,
 * and writes 1 (copied) or 0 to hits[p] (may be null).  Batched form of the
 * cache-hit copy of gsa/session.py:111. */
int reuse_rows_batch(int count, const int* src, long long src_stride,
                     int src_ld, const int* flags, int rows, int cols,
                     int* dst, long long dst_stride, int* hits, void* stream);

/* One hierarchy stage's reuse admission and gather in one launch: for scene
 * p < count, flags[2p] = 1 when the support a[p*a_stride + i] differs from
 * the retained snapshot b[p*b_stride + i] for some i < ns (IEEE !=), and
 * flags[2p+1] = 1 when it differs for some i < nq (the query prefix: the
 * session's query is the support's first nq floats); else 0.  When both are
 * 0 the rows src[p*src_stride + i*src_ld + j] go to dst[p*dst_stride +
 * i*cols + j] (i < rows, j < cols) and hits[p] (may be null) is 1, else 0;
 * rows of a miss are left untouched.  Fused, batched form of the two
 * torch.equal checks and the cached-row copy of gsa/session.py:104-114 (one
 * thread-block cluster per scene).  Returns 0, -2 (bad argument), or a
 * cudaError_t. */
int reuse_prefix_batch(int count, const float* a, long long a_stride,
                       const float* b, long long b_stride, long long ns,
                       long long nq, const int* src, long long src_stride,
                       int src_ld, int rows, int cols, int* dst,
                       long long dst_stride, int* flags, int* hits,
                       void* stream);

/* reuse_prefix_batch for `stages` hierarchy stages of the same scenes in
 * one launch (a cluster per stage and scene): stage i compares ns[i] floats
 * of every scene's support (query prefix nq[i]) and copies rows[i] rows of
 * src[i] (scene stride src_stride[i]) to dst[i] (stride dst_stride[i]),
 * writing flags[i] (2*count ints) and hits[i] (count ints or null).  The
 * per-stage arguments are HOST arrays of `stages` (<= 8) entries; a and b
 * (and their strides), src_ld and cols are shared.  A hierarchy step's four
 * reuse checks run in one launch after its radius stages instead of four
 * launches of mostly latency.  No counterpart in the reference (whose
 * session makes these checks per call, gsa/session.py:104-114).  Returns 0,
 * -2 (bad argument), or a cudaError_t. */
int reuse_prefix_stages(int stages, int count, const float* a,
                        long long a_stride, const float* b,
                        long long b_stride, const long long* ns,
                        const long long* nq, const int* const* src,
                        const long long* src_stride, int src_ld,
                        const int* rows, int cols, int* const* dst,
                        const long long* dst_stride, int* const* flags,
                        int* const* hits, void* stream);

/* Total kernel launches this library has issued since it was loaded. */
int launch_counter(unsigned long long* total);

/* No counterpart in the reference.  Reuse-cache lookup that allocates
 * nothing, for callers that cannot allocate device memory at lookup time
 * (a framework allocator that must not be bypassed, loops where
 * cudaMalloc/cudaFree would synchronise the device, a fixed device
 * footprint after start-up).  Same result as coords_mismatch over the pairs
 * (x, saved_x[c]) with nx floats and (q, saved_q[c]) with nq floats followed
 * by reuse_rows: the rows of the first candidate c whose support and query
 * prefix both equal the current ones (IEEE ==) are copied from cached[c]
 * (row stride src_ld) to dst (rows x cols) and c, or -1, is written to *hit.
 * saved_x, saved_q, cached are HOST arrays of count device pointers.  The
 * per-candidate flags live in a fixed 512-byte device array inside the
 * library (held on every GPU that loads it), so count may not exceed 64:
 * larger counts return -4.  A call outside stream capture looks up that
 * array's device address (again on every such call, so a device reset does
 * not leave a stale address); a call during capture reuses the address of
 * the last uncaptured call on that device, so make one call per device
 * before any stream capture.  Calls share the array: calls whose GPU work
 * overlaps race.  Returns 0, -2 (bad argument), -4, or
 * a cudaError_t. */
int reuse_lookup_static(int count, const float* x, long long nx,
                        const float* q, long long nq,
                        const float* const* saved_x,
                        const float* const* saved_q, const int* const* cached,
                        int src_ld, int rows, int cols, int* dst, int* hit,
                        void* stream);

/* One QuerySession admission step in one call (the comparisons and row copy
 * of gsa/session.py:65-71 and :104-114, which the reference runs as one
 * torch.equal plus host synchronisation per candidate): compares every pair
 * as coords_mismatch does (flags: count device ints, 1 = differs), then,
 * when nmemo > 0, copies the rows of the first memo candidate c whose pairs
 * 2c and 2c+1 both match, as reuse_rows does (nmemo <= 64, pairs 0..2*nmemo-1
 * are the memo pairs), then copies the flags to flags_host (count host
 * ints) and waits for the stream.  Up to 64 pairs and 8 MB of compared and
 * copied data run as one thread-block cluster launch, which writes the flags
 * straight into flags_host when that is pinned host memory.  Returns 0, a
 * cudaError_t, or -2. */
int session_lookup(int count, const float* const* a, const float* const* b,
                   const long long* nfloat, int nmemo,
                   const int* const* cached, int src_ld, int rows, int cols,
                   int* dst, int* flags, int* flags_host, void* stream);

/* Farthest-point order of b scenes of n points each (x is [b][n][3]),
 * starting at start[b] (device int[b]); order is device int[b][n].  Ties pick
 * the lowest index; chosen points are never repeated.  Input generator for
 * FPS-ordered supports (FPS itself lives upstream of GSA, in FlashFPS). */
int fps_order(int b, int n, const float* x, const int* start, int* order,
              void* stream);

/* Farthest-point order of one large scene (up to 8 points per resident
 * thread, about 1.2 M points on a B200) with a cooperative grid: the same
 * rule and result as fps_order.  scratch is 64 bytes of device memory, *err
 * (device int) becomes 1 if a grid barrier wait gives up (the order is then
 * incomplete).  start is a host int. */
int fps_order_large(int n, const float* x, int start, int* order,
                    void* scratch, int* err, void* stream);

/* Furthest point sampling with the PointNet++ operator's arguments
 * (furthest_point_sampling_wrapper(b, n, m, points, temp, idx), the op that
 * samples the query levels GSA's networks search): for each of b scenes of n
 * points (x is [b][n][3]) the first m indices of the farthest-point order
 * starting at index 0, into idx ([b][m] device ints).  Rule: the next point
 * is the one with the largest running minimum of the FP32 squared distance
 * ((dx*dx + dy*dy) + dz*dz) (round to nearest, no FMA) to the points chosen
 * so far, ties to the LOWEST index, chosen points never repeat; a NaN
 * distance never lowers a running minimum, so points with a non-finite
 * coordinate stay at +inf and are chosen first, lowest index first.  Scenes of up to 51,200 points keep the running minima in shared
 * memory (one block per scene; temp may be null).  Larger scenes use one
 * cooperative grid each (up to ~1.2 M points) and need temp (device floats,
 * b*n): its first 17 words of each scene's row are the grid's barrier words
 * and error flag, and ((int*)temp)[n*i + 16] != 0 after the stream reaches
 * it means scene i's order is incomplete (a grid barrier wait ran out).
 * Returns 0, a cudaError_t, or -2 for bad arguments.  The reference has no
 * FPS of its own (it sits upstream, in FlashFPS); the rule is the one its
 * FPS-ordered prefixes assume. */
int furthest_point_sample(int b, int n, int m, const float* x, float* temp,
                          int* idx, void* stream);

#ifdef __cplusplus
}
#endif

#endif
