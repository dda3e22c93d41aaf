// IVF plumbing on the device: probe grouping (list-major work items), the
// stable radix sort behind list building and k-means updates, prefix scans,
// and the deterministic fp64 centroid update.
#include "mf_scan.cuh"
#include "mf_ivf.cuh"
#include "mf_timing.cuh"

namespace mf {

namespace {

constexpr int kScanBlock = 1024;
// List tables of up to this many blocks of kScanBlock lists are planned by
// one block (two scans over the table); longer ones by one block per
// kScanBlock lists in two launches.
constexpr int kPlanOneBlock = 2;

// Block-wide exclusive scan (all kScanBlock threads call it). Returns the
// exclusive prefix of v and writes the block total to `total`.
template <typename T>
__device__ T block_exclusive_scan(T v, T* warp_sums, T& total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = lane < nwarps ? warp_sums[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  const T prefix = warp > 0 ? warp_sums[warp - 1] : T(0);
  total = warp_sums[nwarps - 1];
  __syncthreads();
  return prefix + x - v;
}

// Single-CTA exclusive scan of n values; out has n+1 entries.
template <typename TI, typename TO>
__global__ void __launch_bounds__(kScanBlock) exclusive_scan_kernel(const TI* in, int64_t n, TO* out) {
  __shared__ TO sums[32];
  const int64_t chunk = (n + kScanBlock - 1) / kScanBlock;
  const int64_t b = threadIdx.x * chunk;
  const int64_t e = b + chunk < n ? b + chunk : n;
  TO s = 0;
  for (int64_t i = b; i < e; ++i) s += (TO)in[i];
  TO total;
  TO run = block_exclusive_scan<TO>(s, sums, total);
  for (int64_t i = b; i < e; ++i) {
    const TO v = (TO)in[i];
    out[i] = run;
    run += v;
  }
  if (threadIdx.x == 0) out[n] = total;
}

// --------------------------------------------------------------- grouping
__global__ void ivf_count_kernel(const int64_t* __restrict__ probes, int64_t n, int nlist,
                                 const int64_t* __restrict__ list_offsets, int* counts,
                                 float* pd, int64_t* pl, int k, int64_t* pair_counts, int P,
                                 int s0, int s1) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int slot = (int)(i % P);
  if (slot < s0 || slot >= s1) return;
  const int64_t l = probes[i];
  const bool ok = l >= 0 && l < nlist && list_offsets[l + 1] > list_offsets[l];
  if (ok) {
    atomicAdd(&counts[l], 1);
  } else {
    if (pd) {
      for (int t = 0; t < k; ++t) {
        pd[i * k + t] = __int_as_float(0x7f800000);
        pl[i * k + t] = -1;
      }
    }
    if (pair_counts) pair_counts[i] = 0;
  }
}

// With small_max > 0, a list probed by at most small_max queries goes whole to
// items2 (item_total2) as one item; the other lists' groups go to items. The
// choice depends only on a list's query count, so it does not vary between
// runs; both keep the list order.
__global__ void __launch_bounds__(kScanBlock) ivf_plan_kernel(const int* __restrict__ counts,
                                                             int nlist,
                                                             const int32_t* __restrict__ order,
                                                             int* pair_offsets, int2* items,
                                                             int* item_total, int* cursors,
                                                             int group, int2* items2,
                                                             int* item_total2, int small_max) {
  // Lists in tiles of kScanBlock (thread t: list t0 + t), up to kPlanTiles
  // tiles per pass with every load issued before the first scan.
  constexpr int kPlanTiles = 16;
  __shared__ int sums[32];
  const int t = threadIdx.x;
  // pair offsets, in list-id order
  int base = 0;
  for (int p0 = 0; p0 < nlist; p0 += kPlanTiles * kScanBlock) {
    int v[kPlanTiles];
#pragma unroll
    for (int j = 0; j < kPlanTiles; ++j) {
      const int i = p0 + j * kScanBlock + t;
      v[j] = i < nlist ? counts[i] : 0;
    }
#pragma unroll
    for (int j = 0; j < kPlanTiles; ++j) {
      if (p0 + j * kScanBlock >= nlist) break;  // block-uniform
      const int i = p0 + j * kScanBlock + t;
      int tot;
      const int ex = block_exclusive_scan<int>(v[j], sums, tot);
      if (i < nlist) {
        pair_offsets[i] = base + ex;
        cursors[i] = 0;
      }
      base += tot;
    }
  }
  if (t == 0) pair_offsets[nlist] = base;
  // items, in list order
  int run = 0, run2 = 0;
  for (int p0 = 0; p0 < nlist; p0 += kPlanTiles * kScanBlock) {
    int lv[kPlanTiles], cv[kPlanTiles];
#pragma unroll
    for (int j = 0; j < kPlanTiles; ++j) {
      const int i = p0 + j * kScanBlock + t;
      lv[j] = i < nlist ? (order ? order[i] : i) : -1;
    }
#pragma unroll
    for (int j = 0; j < kPlanTiles; ++j) cv[j] = lv[j] >= 0 ? counts[lv[j]] : 0;
#pragma unroll
    for (int j = 0; j < kPlanTiles; ++j) {
      if (p0 + j * kScanBlock >= nlist) break;  // block-uniform
      const int c = cv[j];
      const int ng = (c + group - 1) / group;
      const bool small_list = small_max > 0 && c > 0 && c <= small_max;
      int tot_a, tot_b;
      const int ea = block_exclusive_scan<int>(small_list ? 0 : ng, sums, tot_a);
      const int eb = block_exclusive_scan<int>(small_list ? 1 : 0, sums, tot_b);
      if (small_list)
        items2[run2 + eb] = make_int2(lv[j], 0);
      else
        for (int g = 0; g < ng; ++g) items[run + ea + g] = make_int2(lv[j], g);
      run += tot_a;
      run2 += tot_b;
    }
  }
  if (t == 0) {
    *item_total = run;
    if (item_total2) *item_total2 = run2;
  }
}

// The same plan over many blocks (one list per thread, kScanBlock lists per
// block), for long list tables: ivf_plan_sums_kernel writes each block's
// three totals (pairs in list-id order; tensor-core groups and few-query
// items in list order), then ivf_plan_write_kernel adds the totals of the
// blocks before its own to its block scans. Same output as ivf_plan_kernel.
__device__ __forceinline__ void plan_terms(const int* __restrict__ counts, int nlist,
                                           const int32_t* __restrict__ order, int i, int group,
                                           int small_max, int& cpair, int& lv, int& c, int& ng,
                                           bool& small_list) {
  cpair = i < nlist ? counts[i] : 0;
  lv = i < nlist ? (order ? order[i] : i) : -1;
  c = lv >= 0 ? counts[lv] : 0;
  ng = (c + group - 1) / group;
  small_list = small_max > 0 && c > 0 && c <= small_max;
}

__global__ void __launch_bounds__(kScanBlock) ivf_plan_sums_kernel(
    const int* __restrict__ counts, int nlist, const int32_t* __restrict__ order, int group,
    int small_max, int3* block_sums) {
  __shared__ int sums[32];
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  int cpair, lv, c, ng;
  bool small_list;
  plan_terms(counts, nlist, order, i, group, small_max, cpair, lv, c, ng, small_list);
  int t0, t1, t2;
  block_exclusive_scan<int>(cpair, sums, t0);
  block_exclusive_scan<int>(small_list ? 0 : ng, sums, t1);
  block_exclusive_scan<int>(small_list ? 1 : 0, sums, t2);
  if (threadIdx.x == 0) block_sums[blockIdx.x] = make_int3(t0, t1, t2);
}

__global__ void __launch_bounds__(kScanBlock) ivf_plan_write_kernel(
    const int* __restrict__ counts, int nlist, const int32_t* __restrict__ order,
    const int3* __restrict__ block_sums, int* pair_offsets, int2* items, int* item_total,
    int* cursors, int group, int2* items2, int* item_total2, int small_max) {
  __shared__ int sums[32];
  __shared__ int3 base;
  if (threadIdx.x == 0) {
    int3 b = make_int3(0, 0, 0);
    for (int j = 0; j < (int)blockIdx.x; ++j) {
      const int3 v = block_sums[j];
      b.x += v.x;
      b.y += v.y;
      b.z += v.z;
    }
    base = b;
  }
  __syncthreads();
  const int i = blockIdx.x * kScanBlock + threadIdx.x;
  int cpair, lv, c, ng;
  bool small_list;
  plan_terms(counts, nlist, order, i, group, small_max, cpair, lv, c, ng, small_list);
  int t0, t1, t2;
  const int e0 = block_exclusive_scan<int>(cpair, sums, t0);
  const int ea = block_exclusive_scan<int>(small_list ? 0 : ng, sums, t1);
  const int eb = block_exclusive_scan<int>(small_list ? 1 : 0, sums, t2);
  if (i < nlist) {
    pair_offsets[i] = base.x + e0;
    cursors[i] = 0;
    if (small_list)
      items2[base.z + eb] = make_int2(lv, 0);
    else
      for (int g = 0; g < ng; ++g) items[base.y + ea + g] = make_int2(lv, g);
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) {
    pair_offsets[nlist] = base.x + t0;
    *item_total = base.y + t1;
    if (item_total2) *item_total2 = base.z + t2;
  }
}

__global__ void ivf_scatter_kernel(const int64_t* __restrict__ probes, int64_t n, int nlist,
                                   const int64_t* __restrict__ list_offsets,
                                   const int* __restrict__ pair_offsets, int* cursors,
                                   int* pairs, int P, int s0, int s1) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int slot = (int)(i % P);
  if (slot < s0 || slot >= s1) return;
  const int64_t l = probes[i];
  if (l >= 0 && l < nlist && list_offsets[l + 1] > list_offsets[l]) {
    const int pos = pair_offsets[l] + atomicAdd(&cursors[l], 1);
    pairs[pos] = (int)i;
  }
}

__global__ void lims_kernel(const int64_t* __restrict__ offsets, int64_t nq, int P,
                            int64_t* lims) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q > nq) return;
  lims[q] = offsets[q * P];
}

// ------------------------------------------------------------ radix sort
constexpr int kRadixBits = 8;
constexpr int kRadixBins = 1 << kRadixBits;
constexpr int kRadixTile = 4096;

__global__ void radix_hist_kernel(const uint32_t* __restrict__ keys, int64_t n, int shift,
                                  int nblocks, int* hist) {
  __shared__ int h[kRadixBins];
  for (int i = threadIdx.x; i < kRadixBins; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int64_t b = (int64_t)blockIdx.x * kRadixTile;
  const int64_t e = b + kRadixTile < n ? b + kRadixTile : n;
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x)
    atomicAdd(&h[(keys[i] >> shift) & (kRadixBins - 1)], 1);
  __syncthreads();
  for (int i = threadIdx.x; i < kRadixBins; i += blockDim.x)
    hist[(int64_t)i * nblocks + blockIdx.x] = h[i];
}

// One warp per tile keeps the scatter stable: lanes are ranked among equal
// digits with __match_any_sync, in input order, chunk by chunk.
__global__ void radix_scatter_kernel(const uint32_t* __restrict__ keys_in,
                                     const int32_t* __restrict__ vals_in, int64_t n, int shift,
                                     int nblocks, const int* __restrict__ offsets,
                                     uint32_t* keys_out, int32_t* vals_out) {
  __shared__ int run[kRadixBins];
  const int lane = threadIdx.x;
  for (int i = lane; i < kRadixBins; i += 32) run[i] = offsets[(int64_t)i * nblocks + blockIdx.x];
  __syncwarp();
  const int64_t b = (int64_t)blockIdx.x * kRadixTile;
  const int64_t e = b + kRadixTile < n ? b + kRadixTile : n;
  for (int64_t c = b; c < e; c += 32) {
    const int64_t i = c + lane;
    const bool v = i < e;
    const uint32_t key = v ? keys_in[i] : 0u;
    const int digit = v ? (int)((key >> shift) & (kRadixBins - 1)) : kRadixBins + lane;
    const unsigned int peers = __match_any_sync(0xffffffffu, digit);
    const int rank = __popc(peers & lanemask_lt());
    int base = 0;
    if (v) base = run[digit];
    __syncwarp();
    if (v) {
      const int pos = base + rank;
      keys_out[pos] = key;
      vals_out[pos] = vals_in ? vals_in[i] : (int32_t)i;
      if (rank == __popc(peers) - 1) run[digit] = base + __popc(peers);
    }
    __syncwarp();
  }
}

__global__ void labels_to_keys_kernel(const int64_t* __restrict__ labels, int64_t n,
                                      uint32_t* keys) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) keys[i] = (uint32_t)labels[i];
}

__global__ void histogram_kernel(const int64_t* __restrict__ labels, int64_t n, int nbins,
                                 int* counts) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t l = labels[i];
  if (l >= 0 && l < nbins) atomicAdd(&counts[l], 1);
}

// ------------------------------------------------------------ IVF add
__global__ void ivf_merge_counts_kernel(const int64_t* __restrict__ old_offsets,
                                        const int* __restrict__ new_counts, int nlist,
                                        int64_t* merged) {
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= nlist) return;
  const int64_t oc = old_offsets ? old_offsets[l + 1] - old_offsets[l] : 0;
  merged[l] = oc + new_counts[l];
}

// Copies one row (vector, norm, id) per warp.
__device__ __forceinline__ void copy_row(const float* src, float* dst, int d, int lane) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int j = lane; j < (d >> 2); j += 32) d4[j] = s4[j];
}

__global__ void ivf_copy_old_kernel(const int64_t* __restrict__ old_offsets, int nlist,
                                    const float* __restrict__ old_vecs,
                                    const float* __restrict__ old_norms,
                                    const int64_t* __restrict__ old_ids, int64_t n_old, int d,
                                    const int64_t* __restrict__ new_offsets, float* out_vecs,
                                    float* out_norms, int64_t* out_ids) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= n_old) return;
  int lo = 0, hi = nlist;  // last l with old_offsets[l] <= r
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (old_offsets[mid] <= r) lo = mid; else hi = mid;
  }
  const int64_t dst = new_offsets[lo] + (r - old_offsets[lo]);
  copy_row(old_vecs + r * d, out_vecs + dst * d, d, lane);
  if (lane == 0) {
    out_norms[dst] = old_norms[r];
    out_ids[dst] = old_ids[r];
  }
}

__global__ void ivf_copy_new_kernel(const uint32_t* __restrict__ sorted_labels,
                                    const int32_t* __restrict__ sorted_rows, int64_t n_new,
                                    const int* __restrict__ new_starts,
                                    const int64_t* __restrict__ old_offsets,
                                    const int64_t* __restrict__ new_offsets,
                                    const float* __restrict__ new_vecs,
                                    const float* __restrict__ new_norms,
                                    const int64_t* __restrict__ new_ids, int d,
                                    float* out_vecs, float* out_norms, int64_t* out_ids) {
  const int lane = threadIdx.x & 31;
  const int64_t j = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (j >= n_new) return;
  const int l = (int)sorted_labels[j];
  const int64_t src = sorted_rows[j];
  const int64_t oc = old_offsets ? old_offsets[l + 1] - old_offsets[l] : 0;
  const int64_t dst = new_offsets[l] + oc + (j - new_starts[l]);
  copy_row(new_vecs + src * d, out_vecs + dst * d, d, lane);
  if (lane == 0) {
    out_norms[dst] = new_norms[src];
    out_ids[dst] = new_ids[src];
  }
}

// -------------------------------------------------------- k-means update
// One CTA per cluster sums its rows (in sorted, i.e. input, order) in fp64.
// One block per cluster: the fp64 sum of its rows in a fixed order, then
// either the mean into `centroids` (an empty cluster keeps its centroid) or,
// with `sums` given, the sums themselves (for a reduction over several GPUs).
__global__ void kmeans_update_kernel(const float* __restrict__ x, int d,
                                     const int32_t* __restrict__ sorted_rows,
                                     const int* __restrict__ starts, int nc, float* centroids,
                                     int64_t* counts, double* sums) {
  const int j = blockIdx.x;
  if (j >= nc) return;
  const int b = starts[j];
  const int e = starts[j + 1];
  const int cnt = e - b;
  if (threadIdx.x == 0 && counts) counts[j] = cnt;
  if (cnt == 0 && sums) {
    for (int c = threadIdx.x; c < d; c += blockDim.x) sums[(int64_t)j * d + c] = 0.0;
  }
  if (cnt == 0) return;  // empty cluster keeps its centroid
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    int i = b;
    for (; i + 4 <= e; i += 4) {
      s0 += (double)x[(int64_t)sorted_rows[i] * d + c];
      s1 += (double)x[(int64_t)sorted_rows[i + 1] * d + c];
      s2 += (double)x[(int64_t)sorted_rows[i + 2] * d + c];
      s3 += (double)x[(int64_t)sorted_rows[i + 3] * d + c];
    }
    for (; i < e; ++i) s0 += (double)x[(int64_t)sorted_rows[i] * d + c];
    const double s = (s0 + s1) + (s2 + s3);
    if (sums)
      sums[(int64_t)j * d + c] = s;
    else
      centroids[(int64_t)j * d + c] = (float)(s / (double)cnt);
  }
}

// centroids[j] = sums[j] / counts[j] where counts[j] > 0 (else unchanged).
__global__ void kmeans_apply_kernel(const double* __restrict__ sums,
                                    const int64_t* __restrict__ counts, int64_t nc, int d,
                                    float* centroids) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nc * d) return;
  const int64_t cnt = counts[i / d];
  if (cnt > 0) centroids[i] = (float)(sums[i] / (double)cnt);
}

}  // namespace

// ================================================================= host side
int launch_exclusive_scan_i64(const int64_t* in, int64_t n, int64_t* out, cudaStream_t stream) {
  exclusive_scan_kernel<int64_t, int64_t><<<1, kScanBlock, 0, stream>>>(in, n, out);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_exclusive_scan_i32(const int* in, int64_t n, int* out, cudaStream_t stream) {
  exclusive_scan_kernel<int, int><<<1, kScanBlock, 0, stream>>>(in, n, out);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_lims(const int64_t* offsets, int64_t nq, int P, int64_t* lims, cudaStream_t stream) {
  lims_kernel<<<(unsigned int)ceil_div(nq + 1, 256), 256, 0, stream>>>(offsets, nq, P, lims);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

size_t ivf_groups_bytes(int64_t nq, int nlist, int P) {
  Carver c(nullptr, 0);
  carve_ivf_groups(c, nq, nlist, P);
  return c.used;
}

IvfGroups carve_ivf_groups(Carver& c, int64_t nq, int nlist, int P) {
  IvfGroups g;
  g.counts = c.take<int>(nlist);
  g.cursors = c.take<int>(nlist);
  g.pair_offsets = c.take<int>((size_t)nlist + 1);
  g.pairs = c.take<int>((size_t)nq * P);
  g.items = c.take<int2>((size_t)nq * P);
  g.item_total = c.take<int>(1);
  g.items2 = c.take<int2>((size_t)nq * P);
  g.item_total2 = c.take<int>(1);
  g.counter = c.take<int>(1);
  g.plan_sums = c.take<int3>((size_t)ceil_div(nlist, kScanBlock));
  return g;
}

int run_ivf_groups_ex(const IvfGroups& g, const int64_t* probes, int64_t nq, int P, int nlist,
                      const int64_t* list_offsets, const int32_t* list_order, float* pd,
                      int64_t* pl, int k, int64_t* pair_counts, int group, cudaStream_t stream,
                      int s0, int s1, int small_max) {
  if (s1 < 0) s1 = P;
  const int64_t n = nq * P;
  ScopedTiming tm("ivf_group", stream);
  MF_CUDA(cudaMemsetAsync(g.counts, 0, sizeof(int) * nlist, stream));
  if (n > 0) {
    ivf_count_kernel<<<(unsigned int)ceil_div(n, 256), 256, 0, stream>>>(
        probes, n, nlist, list_offsets, g.counts, pd, pl, k, pair_counts, P, s0, s1);
    MF_LAUNCH_CHECK();
  }
  const int plan_blocks = (int)ceil_div(nlist, kScanBlock);
  if (plan_blocks <= kPlanOneBlock) {
    ivf_plan_kernel<<<1, kScanBlock, 0, stream>>>(g.counts, nlist, list_order, g.pair_offsets,
                                                  g.items, g.item_total, g.cursors, group,
                                                  g.items2, g.item_total2, small_max);
    MF_LAUNCH_CHECK();
  } else {
    ivf_plan_sums_kernel<<<plan_blocks, kScanBlock, 0, stream>>>(g.counts, nlist, list_order,
                                                                 group, small_max, g.plan_sums);
    MF_LAUNCH_CHECK();
    ivf_plan_write_kernel<<<plan_blocks, kScanBlock, 0, stream>>>(
        g.counts, nlist, list_order, g.plan_sums, g.pair_offsets, g.items, g.item_total,
        g.cursors, group, g.items2, g.item_total2, small_max);
    MF_LAUNCH_CHECK();
  }
  if (n > 0) {
    ivf_scatter_kernel<<<(unsigned int)ceil_div(n, 256), 256, 0, stream>>>(
        probes, n, nlist, list_offsets, g.pair_offsets, g.cursors, g.pairs, P, s0, s1);
    MF_LAUNCH_CHECK();
  }
  return MF_OK;
}

int run_ivf_groups(const IvfGroups& g, const int64_t* probes, int64_t nq, int P, int nlist,
                   const int64_t* list_offsets, const int32_t* list_order, int group,
                   cudaStream_t stream) {
  return run_ivf_groups_ex(g, probes, nq, P, nlist, list_offsets, list_order, nullptr, nullptr,
                           0, nullptr, group, stream);
}

// ---- radix sort of (label, row) pairs by label, stable
size_t radix_sort_bytes(int64_t n) {
  Carver c(nullptr, 0);
  const int64_t nblocks = ceil_div(n > 0 ? n : 1, kRadixTile);
  c.take<uint32_t>(n);
  c.take<uint32_t>(n);
  c.take<int32_t>(n);
  c.take<int32_t>(n);
  c.take<int>((size_t)nblocks * kRadixBins + 1);
  c.take<int>((size_t)nblocks * kRadixBins + 1);
  return c.used;
}

int radix_sort_labels(Carver& c, const int64_t* labels, int64_t n, int max_label,
                      uint32_t** sorted_keys, int32_t** sorted_rows, cudaStream_t stream) {
  const int nblocks = (int)ceil_div(n > 0 ? n : 1, kRadixTile);
  uint32_t* k0 = c.take<uint32_t>(n);
  uint32_t* k1 = c.take<uint32_t>(n);
  int32_t* v0 = c.take<int32_t>(n);
  int32_t* v1 = c.take<int32_t>(n);
  int* hist = c.take<int>((size_t)nblocks * kRadixBins + 1);
  int* offs = c.take<int>((size_t)nblocks * kRadixBins + 1);
  if (!c.fits()) return fail(MF_ERR_INVALID_ARGS, "radix sort workspace too small");
  if (n > 0) {
    labels_to_keys_kernel<<<(unsigned int)ceil_div(n, 256), 256, 0, stream>>>(labels, n, k0);
    MF_LAUNCH_CHECK();
  }
  int bits = 0;
  while (bits < 32 && (1ll << bits) <= (long long)max_label) ++bits;
  const int passes = bits == 0 ? 0 : (bits + kRadixBits - 1) / kRadixBits;
  uint32_t* kin = k0;
  uint32_t* kout = k1;
  int32_t* vin = nullptr;
  int32_t* vout = v0;
  for (int p = 0; p < passes && n > 0; ++p) {
    const int shift = p * kRadixBits;
    radix_hist_kernel<<<nblocks, 256, 0, stream>>>(kin, n, shift, nblocks, hist);
    MF_LAUNCH_CHECK();
    MF_TRY(launch_exclusive_scan_i32(hist, (int64_t)nblocks * kRadixBins, offs, stream));
    radix_scatter_kernel<<<nblocks, 32, 0, stream>>>(kin, vin, n, shift, nblocks, offs, kout,
                                                     vout);
    MF_LAUNCH_CHECK();
    kin = kout;
    kout = (kout == k1) ? k0 : k1;
    vin = vout;
    vout = (vout == v0) ? v1 : v0;
  }
  MF_CHECK(vin != nullptr, MF_ERR_ASSERTION, "radix sort ran no pass (n=%lld, max_label=%d)",
           (long long)n, max_label);
  *sorted_keys = kin;
  *sorted_rows = vin;
  return MF_OK;
}

namespace {
__global__ void iota_kernel(int32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (int32_t)i;
}
}  // namespace

int launch_iota_i32(int32_t* out, int64_t n, cudaStream_t stream) {
  if (n <= 0) return MF_OK;
  iota_kernel<<<(unsigned int)ceil_div(n, 256), 256, 0, stream>>>(out, n);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

size_t ivf_add_bytes(int64_t n_new, int nlist) {
  Carver c(nullptr, 0);
  c.take<int>(nlist);                  // new counts
  c.take<int>((size_t)nlist + 1);      // new starts
  c.take<int64_t>(nlist);              // merged counts
  c.used += radix_sort_bytes(n_new) + 256 * 8;
  return c.used;
}

int run_ivf_add(cudaStream_t stream, int nlist, int d, const int64_t* old_offsets,
                const float* old_vecs, const float* old_norms, const int64_t* old_ids,
                int64_t n_old, const float* new_vecs, const float* new_norms,
                const int64_t* new_ids, const int64_t* new_labels, int64_t n_new,
                int64_t* out_offsets, float* out_vecs, float* out_norms, int64_t* out_ids,
                void* ws, size_t ws_bytes) {
  Carver c(ws, ws_bytes);
  int* new_counts = c.take<int>(nlist);
  int* new_starts = c.take<int>((size_t)nlist + 1);
  int64_t* merged = c.take<int64_t>(nlist);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "ivf add workspace too small");
  MF_CUDA(cudaMemsetAsync(new_counts, 0, sizeof(int) * nlist, stream));
  if (n_new > 0) {
    histogram_kernel<<<(unsigned int)ceil_div(n_new, 256), 256, 0, stream>>>(new_labels, n_new,
                                                                            nlist, new_counts);
    MF_LAUNCH_CHECK();
  }
  MF_TRY(launch_exclusive_scan_i32(new_counts, nlist, new_starts, stream));
  ivf_merge_counts_kernel<<<(unsigned int)ceil_div(nlist, 256), 256, 0, stream>>>(
      n_old > 0 ? old_offsets : nullptr, new_counts, nlist, merged);
  MF_LAUNCH_CHECK();
  MF_TRY(launch_exclusive_scan_i64(merged, nlist, out_offsets, stream));
  if (n_old > 0) {
    ivf_copy_old_kernel<<<(unsigned int)ceil_div(n_old, 8), 256, 0, stream>>>(
        old_offsets, nlist, old_vecs, old_norms, old_ids, n_old, d, out_offsets, out_vecs,
        out_norms, out_ids);
    MF_LAUNCH_CHECK();
  }
  if (n_new > 0) {
    uint32_t* sk = nullptr;
    int32_t* sr = nullptr;
    if (nlist == 1) {
      // Every row goes to list 0: the input order is already sorted.
      sk = c.take<uint32_t>(n_new);
      sr = c.take<int32_t>(n_new);
      MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "ivf add workspace too small");
      MF_CUDA(cudaMemsetAsync(sk, 0, sizeof(uint32_t) * n_new, stream));
      MF_TRY(launch_iota_i32(sr, n_new, stream));
    } else {
      MF_TRY(radix_sort_labels(c, new_labels, n_new, nlist - 1, &sk, &sr, stream));
    }
    ivf_copy_new_kernel<<<(unsigned int)ceil_div(n_new, 8), 256, 0, stream>>>(
        sk, sr, n_new, new_starts, n_old > 0 ? old_offsets : nullptr, out_offsets, new_vecs,
        new_norms, new_ids, d, out_vecs, out_norms, out_ids);
    MF_LAUNCH_CHECK();
  }
  return MF_OK;
}

size_t kmeans_update_bytes(int64_t n, int nc) {
  Carver c(nullptr, 0);
  c.take<int>(nc);
  c.take<int>((size_t)nc + 1);
  c.used += radix_sort_bytes(n) + 256 * 8;
  return c.used;
}

int run_kmeans_update(cudaStream_t stream, const float* x, int64_t n, int d,
                      const int64_t* labels, int nc, float* centroids, int64_t* counts, void* ws,
                      size_t ws_bytes, double* sums) {
  Carver c(ws, ws_bytes);
  int* cnt = c.take<int>(nc);
  int* starts = c.take<int>((size_t)nc + 1);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "k-means update workspace too small");
  MF_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int) * nc, stream));
  if (n > 0) {
    histogram_kernel<<<(unsigned int)ceil_div(n, 256), 256, 0, stream>>>(labels, n, nc, cnt);
    MF_LAUNCH_CHECK();
  }
  MF_TRY(launch_exclusive_scan_i32(cnt, nc, starts, stream));
  uint32_t* sk = nullptr;
  int32_t* sr = nullptr;
  if (n > 0) {
    if (nc == 1) {
      sk = c.take<uint32_t>(n);
      sr = c.take<int32_t>(n);
      MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "k-means update workspace too small");
      MF_TRY(launch_iota_i32(sr, n, stream));
    } else {
      MF_TRY(radix_sort_labels(c, labels, n, nc - 1, &sk, &sr, stream));
    }
  }
  const int threads = d >= 256 ? 256 : ((d + 31) / 32) * 32;
  kmeans_update_kernel<<<nc, threads, 0, stream>>>(x, d, sr, starts, nc, centroids, counts, sums);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_kmeans_apply(const double* sums, const int64_t* counts, int nc, int d, float* centroids,
                        cudaStream_t stream) {
  const int64_t total = (int64_t)nc * d;
  if (total <= 0) return MF_OK;
  kmeans_apply_kernel<<<(unsigned int)ceil_div(total, 256), 256, 0, stream>>>(sums, counts, nc, d,
                                                                              centroids);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

}  // namespace mf
