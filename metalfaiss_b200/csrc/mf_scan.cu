// Slab-scan kernels (SIMT, sm_100a): fused distance tile + per-query warp
// top-k, and the range-search count/fill epilogues. See mf_scan.cuh.
#include "mf_scan.cuh"
#include "mf_timing.cuh"
#include "mf_topk.cuh"

#include <mutex>

namespace mf {

namespace {

template <int METRIC>
__device__ __forceinline__ void accum_tile(float (&acc)[4][4], const float4 (&xv)[4],
                                           const float4 (&qv)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = acc[i][j];
      if (METRIC == MF_METRIC_L2 || METRIC == MF_METRIC_INNER_PRODUCT) {
        a = fmaf(xv[i].x, qv[j].x, a);
        a = fmaf(xv[i].y, qv[j].y, a);
        a = fmaf(xv[i].z, qv[j].z, a);
        a = fmaf(xv[i].w, qv[j].w, a);
      } else if (METRIC == MF_METRIC_L1) {
        a += fabsf(xv[i].x - qv[j].x);
        a += fabsf(xv[i].y - qv[j].y);
        a += fabsf(xv[i].z - qv[j].z);
        a += fabsf(xv[i].w - qv[j].w);
      } else {
        a = fmaxf(a, fabsf(xv[i].x - qv[j].x));
        a = fmaxf(a, fabsf(xv[i].y - qv[j].y));
        a = fmaxf(a, fabsf(xv[i].z - qv[j].z));
        a = fmaxf(a, fabsf(xv[i].w - qv[j].w));
      }
      acc[i][j] = a;
    }
  }
}

struct ScanSmemLayout {
  static constexpr size_t xs_bytes = size_t(kScanStages) * kScanTR * kScanXS * 4;
  static constexpr size_t qs_bytes = size_t(kScanStages) * kScanTQ * kScanXS * 4;
  static constexpr size_t meta_bytes = kScanTQ * (8 + 8 + 4 + 4);
  static size_t bytes(int epi, int kcap) {
    size_t b = xs_bytes + qs_bytes + meta_bytes;
    if (epi == kEpiTopK) b += size_t(kScanTQ) * (kcap + 32) * 8;
    return b;
  }
};

template <int METRIC, int KCAP, int EPI>
__global__ void __launch_bounds__(kScanThreads) scan_kernel(const ScanArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* xs = reinterpret_cast<float*>(smem_raw);
  float* qs = xs + kScanStages * kScanTR * kScanXS;
  long long* s_qout = reinterpret_cast<long long*>(qs + kScanStages * kScanTQ * kScanXS);
  long long* s_off = s_qout + kScanTQ;
  int* s_qrow = reinterpret_cast<int*>(s_off + kScanTQ);
  float* s_qn = reinterpret_cast<float*>(s_qrow + kScanTQ);
  unsigned long long* lists = reinterpret_cast<unsigned long long*>(s_qn + kScanTQ);
  unsigned long long* bufs = lists + kScanTQ * KCAP;

  __shared__ int s_item;
  __shared__ long long s_rb, s_re;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int d = a.d;
  const int k = a.k;
  const int nchunks = (d + kScanDC - 1) / kScanDC;

  for (;;) {
    if (tid == 0) s_item = atomicAdd(a.counter, 1);
    __syncthreads();
    const int item = s_item;
    const int total = a.flat ? a.nqt * a.P : *a.item_total;
    if (item >= total) break;

    // ---- describe the work item: queries, output slots, row slab
    if (a.flat) {
      const int qt = item % a.nqt;
      const int s = item / a.nqt;
      if (tid < kScanTQ) {
        long long q = (long long)qt * kScanTQ + tid;
        bool v = q < a.nq;
        s_qrow[tid] = v ? (int)q : -1;
        s_qout[tid] = v ? (a.direct ? q : q * a.P + s) : -1;
      }
      if (tid == 0) {
        long long rb = (long long)s * a.rows_per_split;
        long long re = rb + a.rows_per_split;
        s_rb = rb;
        s_re = re < a.nb ? re : a.nb;
      }
    } else {
      const int2 it = a.items[item];
      const int pb = a.pair_offsets[it.x] + it.y * (a.group > 0 ? a.group : kScanTQ);
      const int pe0 = a.pair_offsets[it.x + 1];
      const int pe = pe0 < pb + kScanTQ ? pe0 : pb + kScanTQ;
      if (tid < kScanTQ) {
        int p = pb + tid;
        if (p < pe) {
          int pr = a.pairs[p];
          s_qrow[tid] = pr / a.P;
          s_qout[tid] = pr;
        } else {
          s_qrow[tid] = -1;
          s_qout[tid] = -1;
        }
      }
      if (tid == 0) {
        s_rb = a.list_offsets[it.x];
        const long long re = a.list_offsets[it.x + 1];
        s_re = (a.max_rows > 0 && re - s_rb > a.max_rows) ? s_rb + a.max_rows : re;
      }
    }
    __syncthreads();
    if (tid < kScanTQ) {
      int qr = s_qrow[tid];
      s_qn[tid] = (METRIC == MF_METRIC_L2 && qr >= 0) ? a.qnorms[qr] : 0.0f;
      if (EPI == kEpiFill) s_off[tid] = (qr >= 0) ? a.offsets[s_qout[tid]] : 0;
    }
    __syncthreads();

    const long long rb = s_rb;
    const long long re = s_re;
    const long long nrows = re > rb ? re - rb : 0;
    const int ntiles = (int)((nrows + kScanTR - 1) / kScanTR);
    const int total_it = ntiles * nchunks;
    const bool warp_active = s_qrow[warp * 4] >= 0;

    WarpTopK<KCAP> tk[4];
    long long run[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      run[j] = (EPI == kEpiFill) ? s_off[warp * 4 + j] : 0;
      if (EPI == kEpiTopK) {
        unsigned long long bnd = kEmptyKey;
        const int qr = s_qrow[warp * 4 + j];
        if (a.bound && qr >= 0) bnd = bound_key(a.bound[qr]);
        tk[j].init(lists + (warp * 4 + j) * KCAP, bufs + (warp * 4 + j) * 32, k, lane, bnd);
      }
    }

    auto load_stage = [&](int it, int stage) {
      const int t = it / nchunks;
      const int c = it - t * nchunks;
      const long long r0 = rb + (long long)t * kScanTR;
      float* xdst = xs + stage * kScanTR * kScanXS;
#pragma unroll
      for (int s = tid; s < kScanTR * 8; s += kScanThreads) {
        const int row = s >> 3;
        const int part = s & 7;
        const long long grow = r0 + row;
        const int col = c * kScanDC + part * 4;
        const bool v = grow < re && col < d;
        const float* src = v ? a.xb + grow * d + col : a.xb;
        cp_async16(xdst + row * kScanXS + part * 4, src, v);
      }
      {
        const int i = tid >> 3;
        const int part = tid & 7;
        const int qr = s_qrow[i];
        const int col = c * kScanDC + part * 4;
        const bool v = qr >= 0 && col < d;
        const float* src = v ? a.xq + (long long)qr * d + col : a.xq;
        cp_async16(qs + stage * kScanTQ * kScanXS + i * kScanXS + part * 4, src, v);
      }
    };

    float acc[4][4];
#pragma unroll
    for (int s = 0; s < kScanStages - 1; ++s) {
      if (s < total_it) load_stage(s, s);
      cp_async_commit();
    }
    for (int it = 0; it < total_it; ++it) {
      const int stage = it % kScanStages;
      const int t = it / nchunks;
      const int c = it - t * nchunks;
      cp_async_wait<kScanStages - 2>();
      __syncthreads();
      {
        const int nit = it + kScanStages - 1;
        if (nit < total_it) load_stage(nit, nit % kScanStages);
        cp_async_commit();
      }
      if (c == 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
      }
      if (warp_active) {
        const float* X = xs + stage * kScanTR * kScanXS + lane * kScanXS;
        const float* Qp = qs + stage * kScanTQ * kScanXS + (warp * 4) * kScanXS;
#pragma unroll
        for (int kk = 0; kk < kScanDC; kk += 4) {
          float4 xv[4], qv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            xv[i] = *reinterpret_cast<const float4*>(X + i * 32 * kScanXS + kk);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            qv[j] = *reinterpret_cast<const float4*>(Qp + j * kScanXS + kk);
          accum_tile<METRIC>(acc, xv, qv);
        }
      }
      if (c == nchunks - 1 && warp_active) {
        // ---- epilogue: distances of this tile, fed to the per-query selection
        const long long r0 = rb + (long long)t * kScanTR;
        float xn[4];
        bool rv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          long long r = r0 + lane + 32 * i;
          rv[i] = r < re;
          xn[i] = (METRIC == MF_METRIC_L2 && rv[i]) ? a.xnorms[r] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int qi = warp * 4 + j;
          if (s_qrow[qi] < 0) continue;
          const float qnj = s_qn[qi];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const long long r = r0 + lane + 32 * i;
            float dist;
            if (METRIC == MF_METRIC_L2) dist = l2_from_dot(qnj, xn[i], acc[i][j]);
            else if (METRIC == MF_METRIC_INNER_PRODUCT) dist = -acc[i][j];
            else dist = acc[i][j];
            if (EPI == kEpiTopK) {
              tk[j].offer(rv[i] ? make_key(dist, (unsigned int)r) : kEmptyKey, k, lane);
            } else {
              const bool pass = rv[i] && dist <= a.radius;
              const unsigned int m = __ballot_sync(0xffffffffu, pass);
              if (EPI == kEpiFill && pass) {
                const long long pos = run[j] + __popc(m & lanemask_lt());
                a.out_d[pos] = dist;
                a.out_l[pos] = a.ids ? a.ids[r] : r;
              }
              run[j] += __popc(m);
            }
          }
        }
      }
    }
    cp_async_wait<0>();

    // ---- finish the item
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int qi = warp * 4 + j;
      if (s_qrow[qi] < 0) continue;
      const long long slot = s_qout[qi];
      if (EPI == kEpiTopK) {
        tk[j].flush(k, lane);
        for (int t = lane; t < k; t += 32) {
          const unsigned long long key = tk[j].list[t];
          float dv;
          long long lv;
          if (key == kEmptyKey) {
            dv = __int_as_float(0x7f800000);
            lv = -1;
          } else {
            dv = key_dist(key);
            const unsigned int pos = key_index(key);
            lv = a.ids ? a.ids[pos] : (long long)pos;
          }
          a.out_d[slot * k + t] = dv;
          a.out_l[slot * k + t] = lv;
        }
      } else if (EPI == kEpiCount) {
        if (lane == 0) a.counts[slot] = run[j];
      }
    }
    __syncthreads();
  }
}

// Slot j of part p of query q sits at q * qs + p * ps + j (qs, ps in elements,
// one pair for the distances and one for the labels); its key's index is
// p * k_in + j whatever the layout, so equal distances resolve alike.
struct MergeLayout {
  long long d_qs, d_ps, l_qs, l_ps;
};

template <int KCAP>
__global__ void __launch_bounds__(256) merge_kernel(const float* __restrict__ pd,
                                                    const int64_t* __restrict__ pl, int64_t nq,
                                                    int parts, int k_in, int k, MergeLayout ml,
                                                    float* D, int64_t* L) {
  __shared__ unsigned long long lists[8][KCAP];
  __shared__ unsigned long long bufs[8][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long long q = (long long)blockIdx.x * 8 + warp;
  if (q >= nq) return;
  WarpTopK<KCAP> tk;
  tk.init(lists[warp], bufs[warp], k, lane);
  const int total = parts * k_in;
  const float* qd = pd + q * ml.d_qs;
  const int64_t* ql = pl + q * ml.l_qs;
  for (int c0 = 0; c0 < total; c0 += 32) {
    const int c = c0 + lane;
    unsigned long long key = kEmptyKey;
    if (c < total) {
      const int p = c / k_in, j = c - p * k_in;
      if (ql[p * ml.l_ps + j] >= 0) key = make_key(qd[p * ml.d_ps + j], (unsigned int)c);
    }
    tk.offer(key, k, lane);
  }
  tk.flush(k, lane);
  for (int t = lane; t < k; t += 32) {
    const unsigned long long key = tk.list[t];
    if (key == kEmptyKey) {
      D[q * k + t] = __int_as_float(0x7f800000);
      L[q * k + t] = -1;
    } else {
      D[q * k + t] = key_dist(key);
      const int c = (int)key_index(key);
      const int p = c / k_in;
      L[q * k + t] = ql[p * ml.l_ps + (c - p * k_in)];
    }
  }
}

// One warp per query over its row of the distance matrix: the k smallest
// (distance, row) keys, as the fused top-k keeps them.
template <int KCAP>
__global__ void __launch_bounds__(256) dmat_select_kernel(const float* __restrict__ dmat, int64_t ld,
                                                          int64_t nq, int64_t nb, int k,
                                                          const int64_t* __restrict__ ids,
                                                          float* D, int64_t* L) {
  __shared__ unsigned long long lists[8][KCAP];
  __shared__ unsigned long long bufs[8][32];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long long q = (long long)blockIdx.x * 8 + warp;
  if (q >= nq) return;
  WarpTopK<KCAP> tk;
  tk.init(lists[warp], bufs[warp], k, lane);
  const float* row = dmat + q * ld;
  // 128 columns per step, four per lane (ld is a multiple of 128, so a step
  // that starts below nb stays in the row), four steps loaded at once so
  // their reads overlap; a step offers its keys only when some lane holds a
  // distance <= the current k-th (a superset of the keys below it)
  constexpr int kSteps = 4;
  for (long long c0 = 0; c0 < nb; c0 += 128 * kSteps) {
    float4 v[kSteps];
#pragma unroll
    for (int u = 0; u < kSteps; ++u) {
      const long long cu = c0 + 128 * u;  // warp-uniform
      v[u] = cu < nb ? __ldcs(reinterpret_cast<const float4*>(row + cu + 4 * lane))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kSteps; ++u) {
      const long long c = c0 + 128 * u + 4 * lane;
      const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      const float thr_d = tk.thr == kEmptyKey ? __int_as_float(0x7f800000) : key_dist(tk.thr);
      bool any = false;
#pragma unroll
      for (int j = 0; j < 4; ++j) any |= (c + j < nb) && e[j] <= thr_d;
      if (!__any_sync(0xffffffffu, any)) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tk.offer(c + j < nb ? make_key(e[j], (unsigned int)(c + j)) : kEmptyKey, k, lane);
    }
  }
  tk.flush(k, lane);
  for (int t = lane; t < k; t += 32) {
    const unsigned long long key = tk.list[t];
    if (key == kEmptyKey) {
      D[q * k + t] = __int_as_float(0x7f800000);
      L[q * k + t] = -1;
    } else {
      D[q * k + t] = key_dist(key);
      const unsigned int pos = key_index(key);
      L[q * k + t] = ids ? ids[pos] : (int64_t)pos;
    }
  }
}

__global__ void map_ids_kernel(const int64_t* __restrict__ ids, int64_t* labels, int64_t n) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t p = labels[i];
  if (p >= 0) labels[i] = ids[p];
}

__global__ void extract_bound_kernel(const float* __restrict__ pd, int64_t nq, int P, int k,
                                     float* bound) {
  const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (q < nq) bound[q] = pd[(q * P) * k + k - 1];
}

__global__ void norms_kernel(const float* __restrict__ x, int64_t n, int d, float* norms) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  const float* xr = x + row * d;
  float s = 0.0f;
  for (int j = lane; j < d; j += 32) s = fmaf(xr[j], xr[j], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) norms[row] = s;
}

// ----------------------------------------------------------- kernel table
typedef void (*ScanFn)(const ScanArgs);

template <int METRIC>
ScanFn pick_topk(int kcap) {
  switch (kcap) {
    case 32: return scan_kernel<METRIC, 32, kEpiTopK>;
    case 64: return scan_kernel<METRIC, 64, kEpiTopK>;
    case 128: return scan_kernel<METRIC, 128, kEpiTopK>;
    case 256: return scan_kernel<METRIC, 256, kEpiTopK>;
  }
  return nullptr;
}

template <int METRIC>
ScanFn pick(int epi, int kcap) {
  if (epi == kEpiTopK) return pick_topk<METRIC>(kcap);
  if (epi == kEpiCount) return scan_kernel<METRIC, 32, kEpiCount>;
  return scan_kernel<METRIC, 32, kEpiFill>;
}

ScanFn pick_scan(int metric, int epi, int kcap) {
  switch (metric) {
    case MF_METRIC_L2: return pick<MF_METRIC_L2>(epi, kcap);
    case MF_METRIC_INNER_PRODUCT: return pick<MF_METRIC_INNER_PRODUCT>(epi, kcap);
    case MF_METRIC_L1: return pick<MF_METRIC_L1>(epi, kcap);
    case MF_METRIC_LINF: return pick<MF_METRIC_LINF>(epi, kcap);
  }
  return nullptr;
}

constexpr int kMaxDevices = 64;
constexpr int kNumMetric = 4, kNumEpi = 3, kNumKcap = 4;
std::mutex g_attr_mu;
int g_occ[kMaxDevices][kNumMetric][kNumEpi][kNumKcap];  // 0 = unknown

int kcap_slot(int kcap) { return kcap == 32 ? 0 : kcap == 64 ? 1 : kcap == 128 ? 2 : 3; }

// Blocks per SM for an instantiation; sets its shared-memory limit on first use.
int scan_occupancy(int device, int metric, int epi, int kcap, ScanFn fn, size_t smem) {
  if (device < 0 || device >= kMaxDevices) return 1;
  std::lock_guard<std::mutex> lk(g_attr_mu);
  int& slot = g_occ[device][metric][epi][kcap_slot(kcap)];
  if (slot == 0) {
    if (cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return -1;
    int blocks = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, kScanThreads, smem) !=
        cudaSuccess)
      return -1;
    slot = blocks > 0 ? blocks : 1;
  }
  return slot;
}

}  // namespace

int scan_kcap(int k) {
  if (k <= 32) return 32;
  if (k <= 64) return 64;
  if (k <= 128) return 128;
  if (k <= 256) return 256;
  return 0;
}

int launch_scan(const ScanArgs& a, int metric, int epi, int64_t total_items, int device,
                cudaStream_t stream) {
  const int kcap = epi == kEpiTopK ? scan_kcap(a.k) : 32;
  MF_CHECK(kcap != 0, MF_ERR_INVALID_ARGS, "k=%d exceeds the supported maximum %d", a.k, kMaxK);
  ScanFn fn = pick_scan(metric, epi, kcap);
  MF_CHECK(fn != nullptr, MF_ERR_METRIC, "unsupported metric %d", metric);
  const size_t smem = ScanSmemLayout::bytes(epi, kcap);
  const int occ = scan_occupancy(device, metric, epi, kcap, fn, smem);
  MF_CHECK(occ > 0, MF_ERR_CUDA, "could not configure the scan kernel (smem %zu)", smem);
  if (total_items <= 0) return MF_OK;
  long long grid = (long long)num_sms(device) * occ;
  if (grid > total_items) grid = total_items;
  MF_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(int), stream));
  ScopedTiming tm(epi == kEpiTopK
                      ? (a.flat ? "scan_topk_flat"
                                : (a.max_rows > 0 ? "scan_topk_ivf_bound"
                                                  : (a.group > 0 ? "scan_topk_ivf_small"
                                                                 : "scan_topk_ivf")))
                      : "scan_range",
                  stream);
  fn<<<(unsigned int)grid, kScanThreads, smem, stream>>>(a);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_norms(const float* x, int64_t n, int d, float* norms, cudaStream_t stream) {
  if (n <= 0) return MF_OK;
  const int warps = 8;
  const long long grid = ceil_div(n, warps);
  norms_kernel<<<(unsigned int)grid, warps * 32, 0, stream>>>(x, n, d, norms);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_extract_bound(const float* pd, int64_t nq, int P, int k, float* bound,
                         cudaStream_t stream) {
  if (nq <= 0) return MF_OK;
  extract_bound_kernel<<<(unsigned int)ceil_div(nq, 256), 256, 0, stream>>>(pd, nq, P, k, bound);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

// One warp per query: the k-th distance of slot 0 plus a margin that covers
// the difference between two engines' roundings of the same distance. Both
// the SIMT fp32 dot (error <= (d-1) u sum|q_i x_i|, u = 2^-24) and the 3xTF32
// tensor-core dot stay within (d + 32) 2^-22 (|q|^2 + |x|^2) / 2 of the exact
// value, so (d + 32) 2^-21 (qn + max xn) over the rows the bound came from
// bounds their difference with room to spare.
__global__ void extract_bound_slack_kernel(const float* __restrict__ pd, int64_t nq, int P, int k,
                                           const int64_t* __restrict__ probes,
                                           const int64_t* __restrict__ list_offsets,
                                           const float* __restrict__ list_norms,
                                           const float* __restrict__ qnorms, int64_t max_rows,
                                           int d, float* bound) {
  const long long q = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (q >= nq) return;
  const float kth = pd[(q * P) * k + k - 1];
  const long long l = probes[q * P];
  float xmax = 0.0f;
  if (l >= 0) {
    const long long rb = list_offsets[l];
    long long re = list_offsets[l + 1];
    if (re - rb > max_rows) re = rb + max_rows;
    for (long long r = rb + lane; r < re; r += 32) xmax = fmaxf(xmax, list_norms[r]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) xmax = fmaxf(xmax, __shfl_xor_sync(0xffffffffu, xmax, o));
  if (lane == 0) {
    const float gamma = (float)(d + 32) * 4.76837158203125e-07f;  // (d + 32) * 2^-21
    bound[q] = kth + gamma * (qnorms[q] + xmax);  // +inf stays +inf
  }
}

int launch_extract_bound_slack(const float* pd, int64_t nq, int P, int k, const int64_t* probes,
                               const int64_t* list_offsets, const float* list_norms,
                               const float* qnorms, int64_t max_rows, int d, float* bound,
                               cudaStream_t stream) {
  if (nq <= 0) return MF_OK;
  extract_bound_slack_kernel<<<(unsigned int)ceil_div(nq * 32, 256), 256, 0, stream>>>(
      pd, nq, P, k, probes, list_offsets, list_norms, qnorms, max_rows, d, bound);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_map_ids(const int64_t* ids, int64_t* labels, int64_t n, cudaStream_t stream) {
  if (n <= 0) return MF_OK;
  map_ids_kernel<<<(unsigned int)ceil_div(n, 256), 256, 0, stream>>>(ids, labels, n);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_dmat_select(const float* dmat, int64_t ld, int64_t nq, int64_t nb, int k,
                       const int64_t* ids, float* D, int64_t* I, cudaStream_t stream) {
  if (nq <= 0) return MF_OK;
  ScopedTiming tm("dmat_select", stream);
  dmat_select_kernel<32><<<(unsigned int)ceil_div(nq, 8), 256, 0, stream>>>(dmat, ld, nq, nb, k,
                                                                            ids, D, I);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_merge_strided(const float* pd, int64_t d_qs, int64_t d_ps, const int64_t* pl,
                         int64_t l_qs, int64_t l_ps, int64_t nq, int parts, int k_in, int k,
                         float* d, int64_t* l, cudaStream_t stream) {
  if (nq <= 0 || k <= 0) return MF_OK;
  const int kcap = scan_kcap(k);
  MF_CHECK(kcap != 0, MF_ERR_INVALID_ARGS, "k=%d exceeds the supported maximum %d", k, kMaxK);
  MF_CHECK((long long)parts * k_in < (1ll << 31), MF_ERR_INVALID_ARGS,
           "parts*k_in too large for one merge");
  const MergeLayout ml{d_qs, d_ps, l_qs, l_ps};
  const long long grid = ceil_div(nq, 8);
  ScopedTiming tm("merge", stream);
  switch (kcap) {
    case 32: merge_kernel<32><<<(unsigned int)grid, 256, 0, stream>>>(pd, pl, nq, parts, k_in, k, ml, d, l); break;
    case 64: merge_kernel<64><<<(unsigned int)grid, 256, 0, stream>>>(pd, pl, nq, parts, k_in, k, ml, d, l); break;
    case 128: merge_kernel<128><<<(unsigned int)grid, 256, 0, stream>>>(pd, pl, nq, parts, k_in, k, ml, d, l); break;
    default: merge_kernel<256><<<(unsigned int)grid, 256, 0, stream>>>(pd, pl, nq, parts, k_in, k, ml, d, l); break;
  }
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_merge(const float* pd, const int64_t* pl, int64_t nq, int parts, int k_in, int k,
                 float* d, int64_t* l, cudaStream_t stream) {
  const int64_t qs = (int64_t)parts * k_in;
  return launch_merge_strided(pd, qs, k_in, pl, qs, k_in, nq, parts, k_in, k, d, l, stream);
}

// ------------------------------------------------------------- flat search
namespace {
// Tensor-core flat searches whose rows (fp32 + tf32 residual) pass this size
// are cut into row splits of about this size, taken split-major: the CTAs
// working at the same time scan the same split for different query tiles, so
// its rows come from HBM about once and from L2 for the other query tiles
// (equal runs per CTA would stream the whole database once per query tile).
constexpr long long kFlatSplitBytes = 64ll << 20;

void plan_splits(FlatPlan& p, int64_t nq, int64_t nb, int d, int k, int device, int tq,
                 int per_sm) {
  p.nqt = (int)ceil_div(nq, tq);
  if (per_sm == 0 && p.nqt > 1 && (long long)nb * 8 * d > kFlatSplitBytes) {
    long long s = ceil_div((long long)nb * 8 * d, kFlatSplitBytes);
    long long rps = ceil_div(nb, s);
    rps = ceil_div(rps, kScanTR) * kScanTR;
    s = ceil_div(nb, rps);
    p.splits = (int)s;
    p.rows_per_split = rps;
    p.chunk_tiles = 0;
    p.tiles_per_qt = 0;
    p.chunks = (int)((long long)p.nqt * s);
    (void)k;
    return;
  }
  if (per_sm == 0) {
    // Tensor cores, one persistent CTA per SM: equal runs of tiles, each CTA
    // taking the pieces (cut at query-tile boundaries) of its own run, so no
    // SM waits on another's last item. A query tile's pieces write separate
    // partial slots: as many as the most runs one query tile meets.
    const long long sms = device >= 0 ? num_sms(device) : 148;
    const long long tpq = nb > 0 ? ceil_div(nb, kScanTR) : 1;
    const long long total = (long long)(p.nqt > 0 ? p.nqt : 1) * tpq;
    const long long g0 = total < sms ? total : sms;
    const long long T = ceil_div(total, g0);
    long long pmax = 1;
    for (long long q = 0; q < p.nqt; ++q) {
      const long long c0 = (q * tpq) / T;
      const long long c1 = ((q + 1) * tpq - 1) / T;
      if (c1 - c0 + 1 > pmax) pmax = c1 - c0 + 1;
    }
    p.splits = (int)pmax;
    p.rows_per_split = 0;
    p.chunk_tiles = T;
    p.tiles_per_qt = tpq;
    p.chunks = (int)ceil_div(total, T);
    (void)k;
    return;
  }
  // SIMT: about two waves of resident CTAs (per_sm CTAs per SM); tensor
  // cores (per_sm = 0): about one item per SM, since every split restarts the
  // top-k lists. Each split keeps >= 1 tile.
  const long long sms = device >= 0 ? num_sms(device) : 148;
  const long long target = per_sm > 0 ? 2ll * sms * per_sm : sms;
  long long s = ceil_div(target, p.nqt > 0 ? p.nqt : 1);
  const long long max_s = nb > 0 ? ceil_div(nb, kScanTR) : 1;
  if (s > max_s) s = max_s;
  if (s < 1) s = 1;
  long long rps = ceil_div(nb > 0 ? nb : 1, s);
  rps = ceil_div(rps, kScanTR) * kScanTR;
  s = ceil_div(nb > 0 ? nb : 1, rps);
  p.splits = (int)s;
  p.rows_per_split = rps;
  (void)k;
}
}  // namespace

#ifndef MF_DMAT_MAX_QT
#define MF_DMAT_MAX_QT 64
#endif
// The most query tiles the distance-matrix path takes (a tuning build may change it).
constexpr int64_t kDmatMaxQt = MF_DMAT_MAX_QT;

int64_t flat_dmat_ld(int64_t nq, int64_t nb, int k) {
  // Few query tiles per SM: the fused top-k's pieces each start their lists
  // empty, a cost that does not shrink with the queries (at the coarse step
  // over 16384 centroids, k = 32: 0.24 ms for 1,250 queries and 0.47 ms for
  // 10,000 fused, against 0.59 ms for 10,000 through the matrix).
  if (k < 8 || k > 32 || nq < 2 * (int64_t)tc_group() || nq > kDmatMaxQt * (int64_t)tc_group() ||
      nb <= 0 || nb > (1ll << 24))
    return 0;
  const int64_t ld = (nb + 127) / 128 * 128;
  return nq * ld * 4 <= (2ll << 30) ? ld : 0;
}

FlatPlan plan_flat(int64_t nq, int64_t nb, int d, int k, int device, int tq, bool dmat) {
  const int kcap = scan_kcap(k) ? scan_kcap(k) : 256;
  FlatPlan simt, tc;
  plan_splits(simt, nq, nb, d, k, device, 32, kcap >= 256 ? 1 : (kcap >= 128 ? 2 : 3));
  plan_splits(tc, nq, nb, d, k, device, tc_group(), 0);
  FlatPlan p = tq == 32 ? simt : tc;
  // workspace: the larger of the two engines' needs
  const int max_splits = simt.splits > tc.splits ? simt.splits : tc.splits;
  Carver c(nullptr, 0);
  c.take<float>(nq);                        // query norms
  c.take<int>(1);                           // work counter
  c.take<float>((size_t)nq * max_splits * k);
  c.take<int64_t>((size_t)nq * max_splits * k);
  c.take<float>((size_t)nq * d);            // query tf32 residuals (tensor cores)
  c.take<unsigned int>(nq);                 // pieces' shared k-th distances (tensor cores)
  p.bytes_min = c.used;
  p.dmat_ld = dmat ? flat_dmat_ld(nq, nb, k) : 0;
  if (p.dmat_ld > 0) c.take<float>((size_t)nq * p.dmat_ld);  // the distance matrix
  p.bytes = c.used;
  return p;
}

int run_flat_topk(int device, cudaStream_t stream, const float* xq, int64_t nq, const float* xb,
                  const float* xb_norms, const float* xb_lo, int64_t nb, int d, int metric, int k,
                  const int64_t* ids, float* D, int64_t* I, void* ws, size_t ws_bytes,
                  const float* bound) {
  const bool tc = tc_eligible(metric, d, k, nb) && (xb_lo != nullptr || tc_raw_queries(d, k));
  const FlatPlan p = plan_flat(nq, nb, d, k, device, tc ? tc_group() : 32);
  MF_CHECK(ws_bytes >= p.bytes_min, MF_ERR_INVALID_ARGS,
           "flat search workspace too small: %zu < %zu bytes", ws_bytes, p.bytes_min);
  // carve with the same order as plan_flat (partials sized for either engine)
  FlatPlan other = plan_flat(nq, nb, d, k, device, tc ? 32 : tc_group());
  const int max_splits = p.splits > other.splits ? p.splits : other.splits;
  MF_CHECK(other.bytes == p.bytes, MF_ERR_ASSERTION, "flat plan sizes disagree");
  // the distance-matrix path: tensor cores, no bound, a workspace that holds it
  const bool dm = tc && bound == nullptr && p.dmat_ld > 0 && ws_bytes >= p.bytes &&
                  (metric == MF_METRIC_L2 || metric == MF_METRIC_INNER_PRODUCT);
  Carver c(ws, ws_bytes);
  float* qn = c.take<float>(nq);
  int* counter = c.take<int>(1);
  float* pd = c.take<float>((size_t)nq * max_splits * k);
  int64_t* pl = c.take<int64_t>((size_t)nq * max_splits * k);
  float* q_lo = c.take<float>((size_t)nq * d);
  unsigned int* share = c.take<unsigned int>(nq);
  float* dmat = dm ? c.take<float>((size_t)nq * p.dmat_ld) : nullptr;
  if (metric == MF_METRIC_L2) MF_TRY(launch_norms(xq, nq, d, qn, stream));
  ScanArgs a{};
  a.xq = xq;
  a.qnorms = qn;
  a.xb = xb;
  a.xnorms = xb_norms;
  a.ids = p.splits > 1 ? nullptr : ids;
  a.d = d;
  a.k = k;
  a.nq = nq;
  a.P = p.splits;
  a.flat = 1;
  a.nqt = p.nqt;
  a.nb = nb;
  a.rows_per_split = p.rows_per_split;
  a.chunk_tiles = tc ? p.chunk_tiles : 0;
  a.tiles_per_qt = tc ? p.tiles_per_qt : 0;
  a.counter = counter;
  a.bound = bound;
  a.direct = p.splits > 1 ? 0 : 1;
  a.out_d = p.splits > 1 ? pd : D;
  a.out_l = p.splits > 1 ? pl : I;
  if (dm) {
    // every (query tile x row tile) once, distances to the matrix, then the
    // per-query selection (ties to the lower row, as the fused top-k)
    const bool raw = tc_raw_queries(d, k);
    if (!raw) MF_TRY(launch_tf32_residual(xq, nq, d, q_lo, stream));
    a.dmat = dmat;
    a.dmat_ld = p.dmat_ld;
    a.ids = nullptr;
    a.direct = 1;
    a.out_d = nullptr;
    a.out_l = nullptr;
    MF_TRY(launch_tc_scan(a, metric, raw ? nullptr : q_lo, nq, xb_lo, nb, p.chunks, device,
                          stream));
    return launch_dmat_select(dmat, p.dmat_ld, nq, nb, k, ids, D, I, stream);
  }
  if (tc) {
    const bool raw = tc_raw_queries(d, k);  // else the scan streams (xq, q_lo) tiles
    if (!raw) MF_TRY(launch_tf32_residual(xq, nq, d, q_lo, stream));
    // a query tile meets fewer runs than the widest: its other slots stay empty
    if (p.splits > 1) {
      MF_CUDA(cudaMemsetAsync(pl, 0xff, sizeof(int64_t) * (size_t)nq * p.splits * k, stream));
      // the pieces of a query tile share their k-th distances (none yet)
      MF_CUDA(cudaMemsetAsync(share, 0xff, sizeof(unsigned int) * (size_t)nq, stream));
      a.share = share;
    }
    MF_TRY(launch_tc_scan(a, metric, raw ? nullptr : q_lo, nq, xb_lo, nb, p.chunks, device,
                          stream));
  } else {
    MF_TRY(launch_scan(a, metric, kEpiTopK, (int64_t)p.nqt * p.splits, device, stream));
  }
  if (p.splits > 1) {
    MF_TRY(launch_merge(pd, pl, nq, p.splits, k, k, D, I, stream));
    // Row positions are the merge's tie-break, so ids are mapped last.
    if (ids) MF_TRY(launch_map_ids(ids, I, nq * (int64_t)k, stream));
  }
  return MF_OK;
}

}  // namespace mf
