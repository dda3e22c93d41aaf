// Host-side entry points of mf_ivf.cu used by the C-ABI layer.
#pragma once

#include "mf_scan.cuh"

namespace mf {

int launch_exclusive_scan_i32(const int* in, int64_t n, int* out, cudaStream_t stream);
int launch_lims(const int64_t* offsets, int64_t nq, int P, int64_t* lims, cudaStream_t stream);
int launch_iota_i32(int32_t* out, int64_t n, cudaStream_t stream);

// Grouping that also pre-fills the partial slots (pd/pl, k per slot) or the
// per-pair range counts of pairs whose list is empty or out of range. Only
// probe slots in [s0, s1) take part (s1 < 0: all).
int run_ivf_groups_ex(const IvfGroups& g, const int64_t* probes, int64_t nq, int P, int nlist,
                      const int64_t* list_offsets, const int32_t* list_order, float* pd,
                      int64_t* pl, int k, int64_t* pair_counts, int group, cudaStream_t stream,
                      int s0 = 0, int s1 = -1, int small_max = 0);

size_t radix_sort_bytes(int64_t n);

size_t ivf_add_bytes(int64_t n_new, int nlist);
int run_ivf_add(cudaStream_t stream, int nlist, int d, const int64_t* old_offsets,
                const float* old_vecs, const float* old_norms, const int64_t* old_ids,
                int64_t n_old, const float* new_vecs, const float* new_norms,
                const int64_t* new_ids, const int64_t* new_labels, int64_t n_new,
                int64_t* out_offsets, float* out_vecs, float* out_norms, int64_t* out_ids,
                void* ws, size_t ws_bytes);

size_t kmeans_update_bytes(int64_t n, int nc);
// With sums != NULL, writes the per-cluster fp64 sums (nc x d) instead of
// updating the centroids.
int run_kmeans_update(cudaStream_t stream, const float* x, int64_t n, int d,
                      const int64_t* labels, int nc, float* centroids, int64_t* counts, void* ws,
                      size_t ws_bytes, double* sums = nullptr);
int launch_kmeans_apply(const double* sums, const int64_t* counts, int nc, int d, float* centroids,
                        cudaStream_t stream);

}  // namespace mf
