/*
 * metalfaiss_b200 — C-ABI of the B200 (sm_100a) vector-search hot path.
 *
 * Conventions (every entry point):
 *   - returns an int status: MF_OK (0) or one of the MF_ERR_* codes below; the
 *     message of the last failure on the calling thread is mf_last_error().
 *     Nothing aborts and no C++ exception crosses this boundary.
 *   - `device` is the CUDA ordinal the call runs on; `stream` is a cudaStream_t
 *     (NULL = legacy default stream). Work is stream-ordered; the call returns
 *     once the kernels are enqueued.
 *   - every array pointer is a caller-owned DEVICE pointer, 16-byte aligned;
 *     vectors are row-major fp32 with a row length `d` that is a multiple of 4
 *     (callers pad odd dimensions with zeros, which changes none of the four
 *     metrics). Scratch memory is a caller-provided workspace whose size comes
 *     from the matching *_workspace_size query; the library allocates nothing.
 *     A size query plans for the CURRENT CUDA device (its SM count sets the
 *     work split): make the target device current before asking, or the
 *     search may reject the workspace as too small on a device with more SMs.
 *   - distances follow the reference: L2 is the SQUARED distance clamped at 0,
 *     INNER_PRODUCT is returned NEGATED and ranked ascending like the others.
 *   - empty result slots hold distance +inf and label -1.
 *
 * The reference (MetalFaiss, Python on MLX) has no C library: each entry point
 * below replaces a Python function or a Metal kernel launcher, cited beside it
 * as file:line within the reference project.
 */
#ifndef METALFAISS_B200_H
#define METALFAISS_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MF_API __attribute__((visibility("default")))
#else
#define MF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes 0..14 are ErrorCode of python/metalfaiss/errors.py:13-29. */
enum {
  MF_OK = 0,
  MF_ERR_READONLY = 1,
  MF_ERR_MEMORY = 2,
  MF_ERR_IO = 3,
  MF_ERR_RUNTIME = 4,
  MF_ERR_NOT_IMPLEMENTED = 5,
  MF_ERR_INVALID_ARGS = 6,
  MF_ERR_BAD_STATE = 7,
  MF_ERR_ASSERTION = 8,
  MF_ERR_METRIC = 9,
  MF_ERR_INDEX = 10,
  MF_ERR_THREAD = 11,
  MF_ERR_FILE_NOT_FOUND = 12,
  MF_ERR_PERMISSION = 13,
  MF_ERR_FORMAT = 14,
  MF_ERR_CUDA = 100,    /* a CUDA runtime call failed */
  MF_ERR_TIMEOUT = 101  /* a bounded device-side wait gave up */
};

/* Metric ids: the FAISS integers that python/metalfaiss/unittest/test_metric_type.py:29-40
 * expects (the reference's own enums disagree with each other, python/metalfaiss/metric_type.py:10-21). */
enum {
  MF_METRIC_INNER_PRODUCT = 0,
  MF_METRIC_L2 = 1,
  MF_METRIC_L1 = 2,
  MF_METRIC_LINF = 3
};

/* Library version (major*10000 + minor*100 + patch). */
MF_API int mf_version(void);

/* Message of the last failed call on this thread ("" if none). */
MF_API const char* mf_last_error(void);

/* Largest k (and nprobe) the fused top-k kernels accept. */
MF_API int mf_max_k(void);

/* Which engine mf_flat_search runs for this shape: 1 = the tcgen05 tensor-core
 * scan (3xTF32), 0 = the SIMT fp32 scan. has_residuals says whether xb_lo is
 * passed. Host-only, no device needed. No reference counterpart (the
 * reference has one MLX path, python/metalfaiss/indexflat.py:88-110). */
MF_API int mf_flat_engine(int metric, int d, int k, int64_t nb, int has_residuals);

/* Diagnostic of the fp16 tensor-core arithmetic that the filter search's
 * error bound rests on (not a search call): out = A . B^T with fp16 operands
 * and fp32 accumulation, in the exact instruction form of one of the two
 * filter passes. engine 0 = tcgen05.mma kind::f16 with A in tensor memory and
 * B loaded by TMA (the tensor-core filter pass): A and B are 128 x d, out is
 * 128 x 128, 64 <= d <= 128 with d a multiple of 8. engine 1 = mma.sync
 * m16n8k16 (the few-query filter pass): A is 16 x d, B is 8 x d, out is
 * 16 x 8, d a multiple of 16 up to 1024. A and B are row-major fp16 device
 * arrays, out row-major fp32. No reference counterpart (the reference has no
 * reduced-precision path). */
MF_API int mf_diag_f16_dot(int device, void* stream, int engine, const void* a, const void* b,
                           int d, float* out);

/* tf32 residual of each element: lo = x - x with its 13 low mantissa bits
 * cleared. The tensor cores read fp32 operands as tf32 by that truncation, so
 * (x, lo) is the exact two-term split the 3xTF32 scans consume. Computed once
 * per database at add time (no reference counterpart: the reference computes
 * distances in MLX fp32, python/metalfaiss/distances.py:140-173). */
MF_API int mf_tf32_residual(int device, void* stream, const float* x, int64_t n, int d,
                            float* lo);

/* Squared L2 norm of each row: norms[i] = sum_j x[i,j]^2.
 * Replaces the norms_b term of pairwise_L2sqr, python/metalfaiss/distances.py:163-164,
 * computed once at add time instead of on every search. */
MF_API int mf_vector_norms(int device, void* stream, const float* x, int64_t n, int d,
                    float* norms);

/* ---------------------------------------------------------------- flat kNN */

MF_API int mf_flat_search_workspace_size(int64_t nq, int64_t nb, int d, int metric, int k,
                                  size_t* bytes);

/* Exact kNN of xq (nq,d) against xb (nb,d): distances/labels (nq,k), ascending.
 * labels[i,j] = ids[pos] when ids != NULL, else the row position pos.
 * xb_norms (nb) is required for L2 and ignored otherwise. xb_lo (nb,d), optional,
 * is mf_tf32_residual(xb): when given, L2 / inner-product searches with
 * 32 <= d <= 1024, k <= 32 and nb >= 256 run on the tensor cores (3xTF32),
 * otherwise on the SIMT scan.
 * k is clipped by the caller to nb (python/metalfaiss/utils/sorting.py:66-67); here
 * slots beyond nb are padded (+inf, -1).
 * Replaces FlatIndex.search, python/metalfaiss/indexflat.py:70-110 (pairwise_L2sqr
 * distances.py:140-173, -IP indexflat.py:93, L1/Linf indexflat.py:96-99, mlx_topk
 * utils/sorting.py:39-87, id map indexflat.py:109) and the tuple-returning quantizer
 * search python/metalfaiss/index/flat_index.py:70-121. */
MF_API int mf_flat_search(int device, void* stream, const float* xq, int64_t nq,
                   const float* xb, const float* xb_norms, const float* xb_lo, int64_t nb,
                   int d, int metric, int k, const int64_t* ids, float* distances,
                   int64_t* labels, void* workspace, size_t workspace_bytes);

/* mf_flat_search with bound[q] (nq floats), an upper bound on query q's k-th
 * distance known in advance (e.g. from a subset of the rows plus a rounding
 * margin): rows farther than it are not kept, so few candidates reach the
 * top-k lists from the first tile on. With a valid bound the results equal
 * mf_flat_search's; where fewer than k rows are within bound[q] the slots are
 * padded (+inf, -1). Same workspace as mf_flat_search. Used for the coarse
 * step of an IVF search; no counterpart in the reference. */
MF_API int mf_flat_search_bounded(int device, void* stream, const float* xq, int64_t nq,
                                  const float* xb, const float* xb_norms, const float* xb_lo,
                                  int64_t nb, int d, int metric, int k, const int64_t* ids,
                                  const float* bound, float* distances, int64_t* labels,
                                  void* workspace, size_t workspace_bytes);

/* Size of the fixed device scratch array behind mf_flat_search_noalloc. */
#define MF_NOALLOC_SCRATCH_BYTES (16u << 20)

/* mf_flat_search without a workspace, for callers that cannot allocate device
 * memory: an FFI or plugin host that only passes buffers it already owns, code
 * where cudaMalloc is not allowed or would stall the device, or a process
 * whose device footprint must stay fixed after start-up. No counterpart in the
 * reference (its searches allocate through MLX).
 * Same arguments and results as mf_flat_search minus the workspace. Scratch is
 * one file-scope device array of MF_NOALLOC_SCRATCH_BYTES (16 MiB) that every
 * GPU loading this library holds until exit; a search needing more
 * (mf_flat_search_workspace_size > 16 MiB) returns MF_ERR_INVALID_ARGS
 * without launching. Every call looks up the array's address on `device`
 * (nothing is cached, so a device reset leaves no stale address behind); the
 * first call on a device may load the library's device image there and
 * should come before any stream capture on that device. Nothing is allocated
 * or freed. All calls on a device share the array: calls that
 * overlap on the GPU (other streams, other threads) race and must be
 * serialized by the caller. */
MF_API int mf_flat_search_noalloc(int device, void* stream, const float* xq, int64_t nq,
                                  const float* xb, const float* xb_norms, const float* xb_lo,
                                  int64_t nb, int d, int metric, int k, const int64_t* ids,
                                  float* distances, int64_t* labels);

/* ------------------------------------------------------- binary (Hamming) */

/* Binary vectors of d bits (d a multiple of 8, at most 1024) are stored packed
 * as W = ceil(d / 32) uint32 words per row: bit j is bit j % 32 of word j / 32,
 * padding bits zero. The distance is the Hamming distance, the number of
 * coordinates where two vectors differ, as BinaryFlatIndex.search counts it
 * (python/metalfaiss/index/binary_flat_index.py:79-86). */

/* Packs n rows of d coordinates (uint8, nonzero = 1) into codes (n, W).
 * Replaces the uint8 storage of BinaryFlatIndex.add,
 * python/metalfaiss/index/binary_flat_index.py:27-48. */
MF_API int mf_binary_pack(int device, void* stream, const uint8_t* x, int64_t n, int d,
                          uint32_t* codes);

/* The inverse: codes (n, W) -> x (n, d) of 0/1 bytes
 * (BinaryFlatIndex.reconstruct, python/metalfaiss/unittest/test_binary_flat_index.py:80-96). */
MF_API int mf_binary_unpack(int device, void* stream, const uint32_t* codes, int64_t n, int d,
                            uint8_t* x);

MF_API int mf_binary_flat_search_workspace_size(int64_t nq, int64_t nb, int d, int k,
                                                size_t* bytes);

/* Hamming kNN of xq (nq, W) against xb (nb, W): distances (nq, k) as exact
 * fp32 integers, labels (nq, k) (ids[pos] when ids != NULL), ascending by
 * (distance, row); slots beyond nb are (+inf, -1). k <= 256.
 * Replaces BinaryFlatIndex.search, python/metalfaiss/index/binary_flat_index.py:50-92
 * (a (nq, nb) distance matrix and a full argsort there). */
MF_API int mf_binary_flat_search(int device, void* stream, const uint32_t* xq, int64_t nq,
                                 const uint32_t* xb, int64_t nb, int d, int k,
                                 const int64_t* ids, float* distances, int64_t* labels,
                                 void* workspace, size_t workspace_bytes);

MF_API int mf_binary_range_workspace_size(int64_t nq, int64_t nb, int d, size_t* bytes);

/* Range search in two passes over the same workspace: count writes lims
 * (nq + 1) and *total (the host waits for it); fill writes the (distance,
 * label) pairs with distance <= radius, per query in row order.
 * Replaces BinaryFlatIndex.range_search, python/metalfaiss/index/binary_flat_index.py:94-140. */
MF_API int mf_binary_range_count(int device, void* stream, const uint32_t* xq, int64_t nq,
                                 const uint32_t* xb, int64_t nb, int d, int radius,
                                 int64_t* lims, int64_t* total, void* workspace,
                                 size_t workspace_bytes);
MF_API int mf_binary_range_fill(int device, void* stream, const uint32_t* xq, int64_t nq,
                                const uint32_t* xb, int64_t nb, int d, int radius,
                                const int64_t* lims, const int64_t* ids, float* distances,
                                int64_t* labels, void* workspace, size_t workspace_bytes);

MF_API int mf_binary_ivf_search_workspace_size(int64_t nq, int nprobe, int k, size_t* bytes);

/* Binary IVF: Hamming kNN of xq (nq, W) over the lists in probes (nq, nprobe)
 * int64 (-1: none; nprobe <= 64). Lists are CSR: rows [list_offsets[l],
 * list_offsets[l+1]) of list_codes (rows code_pitch >= W words apart) and
 * list_ids (NULL: row positions); a list holds fewer than 2^26 rows.
 * Candidates are ranked by (distance, probe rank, row in list), the order in
 * which BinaryIVFIndex.search concatenates them
 * (python/metalfaiss/index/binary_ivf_index.py:150-185); empty slots are
 * (+inf, -1) (the reference pads label 0). */
MF_API int mf_binary_ivf_search(int device, void* stream, const uint32_t* xq, int64_t nq,
                                const int64_t* probes, int nprobe, int nlist,
                                const int64_t* list_offsets, const uint32_t* list_codes,
                                int code_pitch, const int64_t* list_ids, int d, int k,
                                float* distances, int64_t* labels, void* workspace,
                                size_t workspace_bytes);

/* ----------------------------------------------------------------- IVFPQ */

/* Product-quantization codes (IVFPQIndex.add / ProductQuantizer.compute_codes,
 * python/metalfaiss/index/ivf_pq_index.py:97-113 and
 * python/metalfaiss/index/product_quantizer.py). x (n, dp) fp32 rows of d
 * coordinates (dp >= d, a multiple of 4); pq_centroids (M, ksub, d / M)
 * fp32, ksub <= 256, d / M <= 32, M <= 64. With centroids (nlist, dp) and
 * labels (n) int64 the residual x - centroids[labels] is encoded (IVFPQ),
 * else x itself. codes: (n, code_pitch) bytes, code m of row r at
 * r * code_pitch + m = argmin_j |pq[m][j] - subvector m|^2 (ties to the lowest
 * j); code_pitch is a multiple of 4 >= M, padding bytes zero. */
MF_API int mf_pq_encode(int device, void* stream, const float* x, int64_t n, int dp, int d,
                        int M, int ksub, const float* pq_centroids, const float* centroids,
                        const int64_t* labels, uint8_t* codes, int code_pitch);

MF_API int mf_ivfpq_search_workspace_size(int64_t nq, int nprobe, int k, size_t* bytes);

/* ADC search of the lists in probes (nq, nprobe) int64 (-1 = none): per
 * (query q, list l), the distance of a row with codes c is
 * sum_m |pq[m][c_m] - (q - centroids[l])_m|^2. The lists are CSR: rows
 * [list_offsets[l], list_offsets[l+1]) of list_codes (rows code_pitch bytes
 * apart) and list_ids. Results (nq, k) ascending, labels = list_ids[row]
 * (row positions when list_ids is NULL), empty slots (+inf, -1).
 * Replaces IVFPQIndex.search, python/metalfaiss/index/ivf_pq_index.py:127-186
 * (one query at a time on the host there; empty probes give (+inf, 0), :170-174). */
MF_API int mf_ivfpq_search_preassigned(int device, void* stream, const float* xq, int64_t nq,
                                       int dp, int d, const int64_t* probes, int nprobe,
                                       int nlist, const float* centroids,
                                       const float* pq_centroids, int M, int ksub,
                                       const int64_t* list_offsets, const uint8_t* list_codes,
                                       int code_pitch, const int64_t* list_ids, int k,
                                       float* distances, int64_t* labels, void* workspace,
                                       size_t workspace_bytes);

/* ---------------------------------------------------------------- IVFFlat */

/* Inverted lists are CSR: list l holds rows [list_offsets[l], list_offsets[l+1])
 * of list_vecs (ntotal,d), with list_norms (ntotal) and list_ids (ntotal);
 * ntotal = list_offsets[nlist] is passed by value (the host knows it).
 * list_lo (ntotal,d), optional, is mf_tf32_residual(list_vecs): when given, the
 * L2 / inner-product scan runs on the tensor cores where the shape allows.
 * list_order (nlist, optional) is a permutation of the list ids giving the order
 * in which the scan takes work (largest lists first balances the SMs). */

MF_API int mf_ivf_search_workspace_size(int64_t nq, int nlist, int nprobe, int d, int metric,
                                 int k, size_t* bytes);

/* IVFFlat search: coarse top-nprobe over the centroids (L2), then the exact
 * top-k over the union of the probed lists under `metric`.
 * Replaces IVFFlatIndex.search, python/metalfaiss/index/ivf_flat_index.py:95-151
 * (coarse step :113, gather :118-135, fused scan ivf_list_topk_l2
 * python/metalfaiss/faissmlx/kernels/ivf_kernels.py:21-122,252-294, merge :211-250,364-379). */
MF_API int mf_ivf_search(int device, void* stream, const float* xq, int64_t nq,
                  const float* centroids, const float* centroid_norms, int nlist,
                  int nprobe, const int64_t* list_offsets, const float* list_vecs,
                  const float* list_norms, const float* list_lo, const int64_t* list_ids,
                  int64_t ntotal, const int32_t* list_order, int d, int metric, int k,
                  float* distances, int64_t* labels, void* workspace,
                  size_t workspace_bytes);

MF_API int mf_ivf_search_preassigned_workspace_size(int64_t nq, int nlist, int nprobe, int d,
                                             int metric, int k, size_t* bytes);

/* The list-scan half of mf_ivf_search with caller-supplied probes (nq,nprobe)
 * (list ids; negative entries are skipped). Replaces the per-query gather + fused
 * kernel loop of python/metalfaiss/index/ivf_flat_index.py:115-151 and the
 * search_preassigned call the reference tests expect
 * (python/metalfaiss/unittest/test_mlx_index.py:64-69). */
MF_API int mf_ivf_search_preassigned(int device, void* stream, const float* xq, int64_t nq,
                              const int64_t* probes, int nprobe, int nlist,
                              const int64_t* list_offsets, const float* list_vecs,
                              const float* list_norms, const float* list_lo,
                              const int64_t* list_ids, int64_t ntotal,
                              const int32_t* list_order, int d, int metric, int k,
                              float* distances, int64_t* labels, void* workspace,
                              size_t workspace_bytes);

/* The two halves of mf_ivf_search_preassigned, for an index whose lists are
 * spread over several GPUs (one process per GPU, each holding some lists):
 *
 * mf_ivf_probe_bound writes bound[q] (nq floats): an upper bound on query q's
 * k-th smallest distance over all of its probed lists, taken from the first
 * rows of its first probe (probes[q*nprobe]), or +inf where this process holds
 * no rows of that list. The minimum of the ranks' bounds (an all-reduce) is a
 * bound for every rank; so is the bound a process computes on a copy of every
 * list's first mf_ivf_bound_rows() rows (the same rows the owner would scan),
 * which spares that all-reduce.
 *
 * mf_ivf_search_bounded is mf_ivf_search_preassigned with that bound given:
 * rows farther than bound[q] are not kept, so a rank's results may hold fewer
 * than k rows (padded +inf, -1); merged over the ranks they are the exact
 * top-k. Replaces the sharded IVF search the reference's multi-GPU tests expect
 * (python/metalfaiss/unittest/test_mlx_multi_gpu.py:86-119). Both take the
 * mf_ivf_search_preassigned_workspace_size workspace. */
/* Rows of a query's nearest list that mf_ivf_probe_bound scans (its first
 * rows, at most this many). A process that holds, for every list, a copy of
 * at least these first rows computes every query's bound by itself. */
MF_API int mf_ivf_bound_rows(void);

MF_API int mf_ivf_probe_bound(int device, void* stream, const float* xq, int64_t nq,
                              const int64_t* probes, int nprobe, int nlist,
                              const int64_t* list_offsets, const float* list_vecs,
                              const float* list_norms, const float* list_lo,
                              const int64_t* list_ids, int64_t ntotal, const int32_t* list_order,
                              int d, int metric, int k, float* bound, void* workspace,
                              size_t workspace_bytes);

MF_API int mf_ivf_search_bounded(int device, void* stream, const float* xq, int64_t nq,
                                 const int64_t* probes, int nprobe, int nlist,
                                 const int64_t* list_offsets, const float* list_vecs,
                                 const float* list_norms, const float* list_lo,
                                 const int64_t* list_ids, int64_t ntotal,
                                 const int32_t* list_order, int d, int metric, int k,
                                 const float* bound, float* distances, int64_t* labels,
                                 void* workspace, size_t workspace_bytes);

/* ------------------------------------------------- IVFFlat filter search (L2)
 *
 * The same search as mf_ivf_search for L2, with the list scan split in two:
 * an fp16 tensor-core pass over residuals against the list centroids keeps,
 * per (query, probed list), up to 2k (16..32) smallest upper bounds on the
 * rows' exact distances (bounds from a rigorous per-pair error bound of the
 * fp16 products), then an exact fp32 refinement computes the distances of
 * every row those bounds cannot exclude (rescanning a list exactly where its
 * kept rows cannot prove that) and selects the top-k. The results are the
 * exact top-k over the probed lists, as mf_ivf_search returns them. Same
 * reference interface as mf_ivf_search
 * (python/metalfaiss/index/ivf_flat_index.py:95-151).
 *
 * The bank: list_f16 (ntotal, d) fp16 = round-to-nearest(s_l (list_vecs row -
 * its list's centroid)), list_rnorms (ntotal) = the squared norms of those
 * fp32 residuals, list_stats (nlist, 4) = per list an upper bound on the
 * residual norms, the largest list_norms entry, the power-of-two scale s_l
 * and the power of two beta_l of the norm extension; list_rn16 (ntotal, 16)
 * fp16 = per row [hi, lo, 0, ...] with hi + lo = beta_l list_rnorms[row] (the
 * tensor-core pass folds the residual norms into its accumulator through
 * them). mf_ivf_filter_bank writes all four (after every add, from the CSR
 * bank and the centroids). */

/* 1 when the filter search takes this shape (d a multiple of 8 in [64, 128],
 * 1 <= k <= 16, ntotal >= 256, the tensor-core engine enabled), else 0. */
MF_API int mf_ivf_filter_eligible(int d, int k, int64_t ntotal);

MF_API int mf_ivf_filter_bank(int device, void* stream, int nlist, int d,
                              const int64_t* list_offsets, const float* list_vecs,
                              const float* list_norms, const float* centroids, int64_t ntotal,
                              void* list_f16, float* list_rnorms, void* list_rn16,
                              float* list_stats);

MF_API int mf_ivf_search_filtered_workspace_size(int64_t nq, int nlist, int nprobe, int d, int k,
                                                 size_t* bytes);

MF_API int mf_ivf_search_filtered(int device, void* stream, const float* xq, int64_t nq,
                                  const float* centroids, const float* centroid_norms, int nlist,
                                  int nprobe, const int64_t* list_offsets, const float* list_vecs,
                                  const float* list_norms, const float* list_lo,
                                  const int64_t* list_ids, int64_t ntotal,
                                  const int32_t* list_order, const void* list_f16,
                                  const float* list_rnorms, const void* list_rn16,
                                  const float* list_stats, int d, int k, float* distances,
                                  int64_t* labels, void* workspace, size_t workspace_bytes);

/* mf_ivf_search_bounded for L2 through the filter search (the lists of one
 * rank of a sharded index, caller-supplied probes and the bound from the
 * ranks' mf_ivf_probe_bound minimum): this rank's exact top-k among rows
 * within bound[q], padded (+inf, -1). */
MF_API int mf_ivf_search_bounded_filtered_workspace_size(int64_t nq, int nlist, int nprobe, int d,
                                                         int k, size_t* bytes);

MF_API int mf_ivf_search_bounded_filtered(int device, void* stream, const float* xq, int64_t nq,
                                          const int64_t* probes, int nprobe, int nlist,
                                          const int64_t* list_offsets, const float* list_vecs,
                                          const float* list_norms, const int64_t* list_ids,
                                          int64_t ntotal, const int32_t* list_order,
                                          const void* list_f16, const float* list_rnorms,
                                          const void* list_rn16, const float* list_stats,
                                          const float* centroids, int d,
                                          int k, const float* bound, float* distances,
                                          int64_t* labels, void* workspace,
                                          size_t workspace_bytes);

/* Lists the filter search's refinement rescanned exactly on `device` since the
 * last reset (a statistic; reset != 0 clears it after reading). */
MF_API int mf_ivf_filter_rescans(int device, int64_t* count, int reset);

/* ----------------------------------------------------------- merge, k-means */

/* Merge `parts` partial top-k lists per query: in (nq, parts, k_in) ascending,
 * out (nq, k). Used for cross-split, cross-list and cross-GPU merges.
 * Replaces device_topk_merge, python/metalfaiss/faissmlx/kernels/ivf_kernels.py:211-250,364-379. */
MF_API int mf_topk_merge(int device, void* stream, const float* part_distances,
                  const int64_t* part_labels, int64_t nq, int parts, int k_in, int k,
                  float* distances, int64_t* labels);

/* mf_topk_merge over any layout of the partial lists: slot j of part p of
 * query q is part_distances[q * dist_query_stride + p * dist_part_stride + j]
 * and part_labels[q * label_query_stride + p * label_part_stride + j]
 * (element strides). Equal distances resolve by (p, j) as in mf_topk_merge,
 * so the result does not depend on the layout. It reads the partials of the
 * processes of a sharded search where an all-gather left them, part-major
 * ((parts, nq, k_in), distances and labels in one buffer per part), without
 * a transposing copy. Replaces the same device_topk_merge
 * (python/metalfaiss/faissmlx/kernels/ivf_kernels.py:211-250). */
MF_API int mf_topk_merge_strided(int device, void* stream, const float* part_distances,
                                 int64_t dist_query_stride, int64_t dist_part_stride,
                                 const int64_t* part_labels, int64_t label_query_stride,
                                 int64_t label_part_stride, int64_t nq, int parts, int k_in,
                                 int k, float* distances, int64_t* labels);

MF_API int mf_kmeans_assign_workspace_size(int64_t n, int nc, int d, size_t* bytes);

/* k-means assignment: labels[i] = argmin_j ||x_i - c_j||^2 (ties: lowest j),
 * min_distances[i] = that squared distance (may be NULL).
 * Replaces python/metalfaiss/clustering/any_clustering.py:105-106 and
 * python/metalfaiss/index/ivf_pq_index.py:66-67. */
MF_API int mf_kmeans_assign(int device, void* stream, const float* x, int64_t n,
                     const float* centroids, const float* centroid_norms, int nc, int d,
                     int64_t* labels, float* min_distances, void* workspace,
                     size_t workspace_bytes);

MF_API int mf_kmeans_update_workspace_size(int64_t n, int nc, int d, size_t* bytes);

/* k-means update: centroids[j] = mean of the rows assigned to j; a cluster with
 * no rows keeps its previous centroid (updated in place). counts (nc) receives
 * the cluster sizes. Sums are accumulated in fp64 in a fixed order (deterministic).
 * Replaces python/metalfaiss/clustering/any_clustering.py:109-120 and
 * python/metalfaiss/index/ivf_pq_index.py:68-78. */
MF_API int mf_kmeans_update(int device, void* stream, const float* x, int64_t n, int d,
                     const int64_t* labels, int nc, float* centroids, int64_t* counts,
                     void* workspace, size_t workspace_bytes);

/* The update split in two for training over several GPUs (each holding a
 * share of the points, centroids replicated): mf_kmeans_sums writes the
 * per-cluster fp64 sums (nc x d) and sizes of this share (same workspace as
 * mf_kmeans_update); after a SUM all-reduce of both, mf_kmeans_apply sets
 * centroids[j] = sums[j] / counts[j], leaving empty clusters unchanged.
 * Replaces the same steps of python/metalfaiss/clustering/any_clustering.py:109-120;
 * the reference trains on one device only. */
MF_API int mf_kmeans_sums(int device, void* stream, const float* x, int64_t n, int d,
                          const int64_t* labels, int nc, double* sums, int64_t* counts,
                          void* workspace, size_t workspace_bytes);
MF_API int mf_kmeans_apply(int device, void* stream, const double* sums, const int64_t* counts,
                           int nc, int d, float* centroids);

/* ------------------------------------------------------------- IVF build */

MF_API int mf_ivf_add_workspace_size(int64_t n_old, int64_t n_new, int nlist, size_t* bytes);

/* Append n_new rows to the CSR lists. new_labels (n_new) are the coarse
 * assignments (mf_kmeans_assign). Output CSR (caller-allocated, n_old + n_new
 * rows) keeps every old row, in order, followed by the new rows of that list in
 * input order (a stable counting sort by list id).
 * Replaces IVFFlatIndex.add, python/metalfaiss/index/ivf_flat_index.py:74-93. */
MF_API int mf_ivf_add(int device, void* stream, int nlist, int d,
               const int64_t* old_offsets, const float* old_vecs,
               const float* old_norms, const int64_t* old_ids, int64_t n_old,
               const float* new_vecs, const float* new_norms, const int64_t* new_ids,
               const int64_t* new_labels, int64_t n_new, int64_t* out_offsets,
               float* out_vecs, float* out_norms, int64_t* out_ids, void* workspace,
               size_t workspace_bytes);

/* ---------------------------------------------------------- range search */

MF_API int mf_flat_range_workspace_size(int64_t nq, int64_t nb, int d, size_t* bytes);

/* Exact range search, first pass: lims (nq+1) gets the prefix sums of the
 * per-query counts of rows with distance <= radius (ascending metrics; for
 * INNER_PRODUCT the distance is -IP like everywhere else). *total receives lims[nq]
 * (a host pointer; the call synchronizes the stream to read it).
 * Replaces Index.range_search, python/metalfaiss/index.py:90-130, without its
 * k=min(100,ntotal) cap (python/metalfaiss/index.py:104). */
MF_API int mf_flat_range_count(int device, void* stream, const float* xq, int64_t nq,
                        const float* xb, const float* xb_norms, int64_t nb, int d,
                        int metric, float radius, int64_t* lims, int64_t* total,
                        void* workspace, size_t workspace_bytes);

/* Second pass: writes the (distance, label) pairs of each query at
 * [lims[q], lims[q+1]) in row order. The workspace must be the one the count
 * pass used, unchanged. */
MF_API int mf_flat_range_fill(int device, void* stream, const float* xq, int64_t nq,
                       const float* xb, const float* xb_norms, int64_t nb, int d,
                       int metric, float radius, const int64_t* ids, const int64_t* lims,
                       float* distances, int64_t* labels, void* workspace,
                       size_t workspace_bytes);

MF_API int mf_ivf_range_workspace_size(int64_t nq, int nlist, int nprobe, int d, size_t* bytes);

/* IVF range search over the probed lists (coarse step as mf_ivf_search), count pass. */
MF_API int mf_ivf_range_count(int device, void* stream, const float* xq, int64_t nq,
                       const float* centroids, const float* centroid_norms, int nlist,
                       int nprobe, const int64_t* list_offsets, const float* list_vecs,
                       const float* list_norms, int d, int metric, float radius,
                       int64_t* lims, int64_t* total, void* workspace,
                       size_t workspace_bytes);

/* IVF range search, fill pass (probe order, then row order within each list). */
MF_API int mf_ivf_range_fill(int device, void* stream, const float* xq, int64_t nq,
                      const float* centroids, const float* centroid_norms, int nlist,
                      int nprobe, const int64_t* list_offsets, const float* list_vecs,
                      const float* list_norms, const int64_t* list_ids, int d,
                      int metric, float radius, const int64_t* lims, float* distances,
                      int64_t* labels, void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------- diagnostics */

/* CUDA-event timing of this library's own launches, per kernel name
 * ("scan_topk", "scan_range", "merge", "ivf_group", "norms"). Replaces the
 * wall-clock median_time harness of python/metalfaiss/benchmarks/run_benchmarks.py:27-44
 * with device-side times. mf_timing_read needs the streams synchronized. */
MF_API int mf_timing_enable(int enable);
MF_API int mf_timing_reset(void);
MF_API int mf_timing_read(const char* kernel, double* total_ms, int64_t* launches);

/* Number of kernels this library has launched in this process (all devices). */
MF_API int64_t mf_launch_count(void);

/* Epilogue warpgroups of the filter search's tensor-core pass: 2 (the
 * default; each takes half of every tile's columns) or 1. Results are the
 * same; for tests and measurements. No reference counterpart. */
MF_API int mf_set_filter_groups(int groups);

/* The filter search sends lists probed by at most `queries` queries (0 to 16;
 * default 16) to its few-query pass and the others to the tensor-core pass.
 * Results are the same; for measurements. No reference counterpart. */
MF_API int mf_set_filter_small_group(int queries);

/* Scan engine for the L2 / inner-product top-k scans: 0 = automatic (tensor
 * cores where the shape allows), 1 = SIMT only, 2 = tensor cores where the
 * shape allows, 3 = as 2 but with the query tile streamed through shared
 * memory even where it fits in tensor memory (d <= 128). Mirrors the
 * reference's kernel switches (python/metalfaiss/faissmlx/flags.py:20-35).
 * Process-wide. */
MF_API int mf_set_scan_engine(int engine);

/* Reads and clears the device-side error word of `device` (MF_ERR_TIMEOUT if a
 * bounded wait in a kernel gave up since the last read, else MF_OK).
 * Synchronizes the device. */
MF_API int mf_device_error(int device, int* code);

#ifdef __cplusplus
}
#endif

#endif /* METALFAISS_B200_H */
