// IVFPQ on the B200: residual product-quantization codes of the inverted
// lists and their asymmetric-distance (ADC) scan, the search of IVFPQIndex
// (python/metalfaiss/index/ivf_pq_index.py:25-192).
//
// A database row x assigned to list l is stored as M one-byte codes: code m
// is the nearest of the ksub (<= 256) centroids of subspace m (dsub = d / M
// coordinates) to the residual (x - c_l) restricted to that subspace
// (ProductQuantizer.compute_codes, python/metalfaiss/index/product_quantizer.py).
// A query q probing list l is scored against each row by
//   sum_m LUT[m][code_m],  LUT[m][j] = |pq[m][j] - (q - c_l)_m|^2
// (IVFPQIndex._adc_lut and search, :115-170): the squared L2 distance of q to
// the row's reconstruction c_l + decode(codes).
//
// Scan: one block of 256 threads per (query, probe) pair. The block forms the
// pair's LUT (M x ksub floats) in shared memory, then its warps take the
// list's rows 32 at a time (one row per lane: its M code bytes in one or a
// few 16-byte loads, M shared-memory lookups), feed per-warp top-k lists, and
// merge them into the pair's k best (distance, row) at the end. The (query,
// probe) partials are merged per query on the device (merge_kernel), then the
// row positions are mapped to ids. Codes are the memory traffic: M bytes per
// row read once per probing query.
#include "mf_scan.cuh"
#include "mf_timing.cuh"
#include "mf_topk.cuh"

namespace mf {
namespace {

constexpr int kPqThreads = 256;
constexpr int kPqWarps = kPqThreads / 32;
constexpr int kPqMaxM = 64;
constexpr int kPqMaxD = 1024;
constexpr int kPqMaxDsub = 32;

struct PqArgs {
  const float* xq;        // (nq, dp)
  const int64_t* probes;  // (nq, P)
  const float* cents;     // (nlist, dp)
  const float* pq;        // (M, ksub, dsub)
  const int64_t* offsets; // (nlist + 1)
  const uint8_t* codes;   // (ntotal, cp): M code bytes per row, rows cp bytes apart
  int64_t nq;
  int P, dp, d, M, cp, ksub, dsub, k, nlist;
  float* out_d;           // (nq, P, k)
  int64_t* out_l;
};

// Residual PQ codes: block (row tile, subspace m); the subspace's centroids
// sit in shared memory, each thread encodes one row: the argmin over j of
// |pq[m][j] - (x - c_label)_m|^2, ties to the lowest j.
__global__ void __launch_bounds__(256)
    pq_encode_kernel(const float* __restrict__ x, int64_t n, int dp, int M, int cp, int ksub,
                     int dsub, const float* __restrict__ pq, const float* __restrict__ cents,
                     const int64_t* __restrict__ labels, uint8_t* __restrict__ codes) {
  extern __shared__ float pq_s[];  // ksub x dsub
  const int m = blockIdx.y;
  for (int i = threadIdx.x; i < ksub * dsub; i += blockDim.x)
    pq_s[i] = pq[(size_t)m * ksub * dsub + i];
  __syncthreads();
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  float res[kPqMaxDsub];
  const float* xr = x + r * dp + m * dsub;
  const int64_t lab = labels ? labels[r] : -1;
  const float* cr = lab >= 0 ? cents + lab * dp + m * dsub : nullptr;
#pragma unroll
  for (int t = 0; t < kPqMaxDsub; ++t)
    res[t] = t < dsub ? xr[t] - (cr ? cr[t] : 0.0f) : 0.0f;
  float best = __int_as_float(0x7f800000);
  int bj = 0;
  for (int j = 0; j < ksub; ++j) {
    const float* c = pq_s + j * dsub;
    float s = 0.0f;
#pragma unroll
    for (int t = 0; t < kPqMaxDsub; ++t) {
      if (t < dsub) {
        const float df = c[t] - res[t];
        s = fmaf(df, df, s);
      }
    }
    if (s < best) {
      best = s;
      bj = j;
    }
  }
  codes[r * cp + m] = (uint8_t)bj;
  if (m == 0)  // the row's padding bytes past M
    for (int p = M; p < cp; ++p) codes[r * cp + p] = 0;
}

template <int KCAP>
__global__ void __launch_bounds__(kPqThreads)
    pq_scan_kernel(const PqArgs a) {
  extern __shared__ unsigned char pq_smem[];
  float* lut = reinterpret_cast<float*>(pq_smem);                     // M x ksub
  float* qres = lut + a.M * a.ksub;                                     // d
  unsigned long long* lists = reinterpret_cast<unsigned long long*>(   // 8 x KCAP
      reinterpret_cast<uintptr_t>(qres + a.d + 1) + 7 & ~uintptr_t(7));
  unsigned long long* bufs = lists + kPqWarps * KCAP;                  // 8 x 32
  const int pair = blockIdx.x;
  const int64_t q = pair / a.P;
  const int64_t l = a.probes[pair];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* od = a.out_d + (size_t)pair * a.k;
  int64_t* ol = a.out_l + (size_t)pair * a.k;
  if (l < 0 || l >= a.nlist) {  // no list: empty slots
    for (int i = threadIdx.x; i < a.k; i += kPqThreads) {
      od[i] = __int_as_float(0x7f800000);
      ol[i] = -1;
    }
    return;
  }
  // the query's residual against the list centroid, then the LUT
  for (int t = threadIdx.x; t < a.d; t += kPqThreads)
    qres[t] = a.xq[q * a.dp + t] - a.cents[l * a.dp + t];
  __syncthreads();
  for (int e = threadIdx.x; e < a.M * a.ksub; e += kPqThreads) {
    const int m = e / a.ksub;
    const int j = e - m * a.ksub;
    const float* c = a.pq + ((size_t)m * a.ksub + j) * a.dsub;
    const float* r = qres + m * a.dsub;
    float s = 0.0f;
    for (int t = 0; t < a.dsub; ++t) {
      const float df = c[t] - r[t];
      s = fmaf(df, df, s);
    }
    lut[e] = s;
  }
  WarpTopK<KCAP> tk;
  tk.init(lists + warp * KCAP, bufs + warp * 32, a.k, lane);
  __syncthreads();
  const int64_t rb = a.offsets[l], re = a.offsets[l + 1];
  const int M = a.M, ksub = a.ksub;
  for (int64_t r0 = rb + 32 * warp; r0 < re; r0 += 32 * kPqWarps) {
    const int64_t row = r0 + lane;
    unsigned long long key = kEmptyKey;
    if (row < re) {
      // the row's codes four at a time (rows are cp = M rounded up to 4 bytes apart)
      const uint32_t* c = reinterpret_cast<const uint32_t*>(a.codes + row * a.cp);
      float s = 0.0f;
      for (int m0 = 0; m0 < M; m0 += 4) {
        const uint32_t w = c[m0 >> 2];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) s += lut[(m0 + i) * ksub + ((w >> (8 * i)) & 0xffu)];
      }
      key = make_key(s, (unsigned int)row);
    }
    tk.offer(key, a.k, lane);
  }
  tk.flush(a.k, lane);
  __syncthreads();
  // warp 0 merges the other warps' lists, 32 keys per offer
  if (warp == 0) {
    for (int w = 1; w < kPqWarps; ++w)
      for (int i = 0; i < a.k; i += 32)
        tk.offer(i + lane < a.k ? lists[w * KCAP + i + lane] : kEmptyKey, a.k, lane);
    tk.flush(a.k, lane);
    for (int i = lane; i < a.k; i += 32) {
      const unsigned long long key = tk.list[i];
      od[i] = key == kEmptyKey ? __int_as_float(0x7f800000) : key_dist(key);
      ol[i] = key == kEmptyKey ? -1 : (int64_t)key_index(key);
    }
  }
}

int pq_kcap(int k) { return k <= 32 ? 32 : (k <= 128 ? 128 : (k <= 256 ? 256 : 0)); }

size_t pq_scan_smem(int M, int ksub, int d, int kcap) {
  return (size_t)M * ksub * 4 + (size_t)(d + 1) * 4 + 8 + (size_t)kPqWarps * (kcap + 32) * 8;
}

int check_pq_shape(int d, int M, int ksub) {
  MF_CHECK(M >= 1 && M <= kPqMaxM && d > 0 && d <= kPqMaxD && d % M == 0, MF_ERR_INVALID_ARGS,
           "PQ shape d=%d M=%d (M in [1, %d] dividing d <= %d)", d, M, kPqMaxM, kPqMaxD);
  MF_CHECK(d / M <= kPqMaxDsub, MF_ERR_INVALID_ARGS, "PQ subspace of %d coordinates (at most %d)",
           d / M, kPqMaxDsub);
  MF_CHECK(ksub >= 1 && ksub <= 256, MF_ERR_INVALID_ARGS, "ksub=%d (1 to 256: one-byte codes)",
           ksub);
  return MF_OK;
}

}  // namespace
}  // namespace mf

using namespace mf;

#define MF_PQ_ENTER(device)                  \
  clear_error();                             \
  DeviceGuard _guard(device);                \
  if (_guard.status != MF_OK) return _guard.status

extern "C" {

int mf_pq_encode(int device, void* stream, const float* x, int64_t n, int dp, int d, int M,
                 int ksub, const float* pq_centroids, const float* centroids,
                 const int64_t* labels, uint8_t* codes, int code_pitch) {
  MF_PQ_ENTER(device);
  MF_TRY(check_pq_shape(d, M, ksub));
  MF_CHECK(dp >= d && dp % 4 == 0, MF_ERR_INVALID_ARGS, "row pitch dp=%d for d=%d", dp, d);
  MF_CHECK(n >= 0, MF_ERR_INVALID_ARGS, "negative n");
  MF_CHECK(code_pitch >= M && code_pitch % 4 == 0, MF_ERR_INVALID_ARGS,
           "code pitch %d (a multiple of 4, at least M=%d)", code_pitch, M);
  if (n == 0) return MF_OK;
  MF_TRY(check_device_ptr(x, "x"));
  MF_TRY(check_device_ptr(pq_centroids, "pq_centroids"));
  MF_TRY(check_device_ptr(codes, "codes"));
  MF_CHECK((centroids == nullptr) == (labels == nullptr), MF_ERR_INVALID_ARGS,
           "centroids and labels go together (residual codes) or not at all");
  MF_TRY(check_device_ptr(centroids, "centroids", true));
  MF_TRY(check_device_ptr(labels, "labels", true));
  const int dsub = d / M;
  dim3 grid((unsigned)ceil_div(n, 256), (unsigned)M);
  pq_encode_kernel<<<grid, 256, (size_t)ksub * dsub * 4, (cudaStream_t)stream>>>(
      x, n, dp, M, code_pitch, ksub, dsub, pq_centroids, centroids, labels, codes);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int mf_ivfpq_search_workspace_size(int64_t nq, int nprobe, int k, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_CHECK(k >= 1 && k <= kMaxK && nprobe >= 1 && nq >= 0, MF_ERR_INVALID_ARGS,
           "k=%d nprobe=%d", k, nprobe);
  Carver c(nullptr, 0);
  c.take<float>((size_t)nq * nprobe * k);
  c.take<int64_t>((size_t)nq * nprobe * k);
  *bytes = c.used;
  return MF_OK;
}

int mf_ivfpq_search_preassigned(int device, void* stream, const float* xq, int64_t nq, int dp,
                                int d, const int64_t* probes, int nprobe, int nlist,
                                const float* centroids, const float* pq_centroids, int M,
                                int ksub, const int64_t* list_offsets, const uint8_t* list_codes,
                                int code_pitch, const int64_t* list_ids, int k, float* distances,
                                int64_t* labels, void* workspace, size_t workspace_bytes) {
  MF_PQ_ENTER(device);
  MF_TRY(check_pq_shape(d, M, ksub));
  MF_CHECK(dp >= d && dp % 4 == 0, MF_ERR_INVALID_ARGS, "row pitch dp=%d for d=%d", dp, d);
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d must be in [1, %d]", k, kMaxK);
  MF_CHECK(nprobe >= 1 && nlist >= 1 && nq >= 0, MF_ERR_INVALID_ARGS, "nprobe=%d nlist=%d",
           nprobe, nlist);
  MF_CHECK(nq * nprobe < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  MF_CHECK(code_pitch >= M && code_pitch % 4 == 0, MF_ERR_INVALID_ARGS,
           "code pitch %d (a multiple of 4, at least M=%d)", code_pitch, M);
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(probes, "probes"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  MF_TRY(check_device_ptr(pq_centroids, "pq_centroids"));
  MF_TRY(check_device_ptr(list_offsets, "list_offsets"));
  MF_TRY(check_device_ptr(list_codes, "list_codes", true));
  MF_TRY(check_device_ptr(list_ids, "list_ids", true));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  float* pd = c.take<float>((size_t)nq * nprobe * k);
  int64_t* pl = c.take<int64_t>((size_t)nq * nprobe * k);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "IVFPQ workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  cudaStream_t st = (cudaStream_t)stream;
  PqArgs a{};
  a.xq = xq;
  a.probes = probes;
  a.cents = centroids;
  a.pq = pq_centroids;
  a.offsets = list_offsets;
  a.codes = list_codes;
  a.nq = nq;
  a.P = nprobe;
  a.dp = dp;
  a.d = d;
  a.M = M;
  a.cp = code_pitch;
  a.ksub = ksub;
  a.dsub = d / M;
  a.k = k;
  a.nlist = nlist;
  a.out_d = pd;
  a.out_l = pl;
  const int kcap = pq_kcap(k);
  const size_t smem = pq_scan_smem(M, ksub, d, kcap);
  MF_CHECK(smem <= 227 * 1024, MF_ERR_INVALID_ARGS, "IVFPQ scan needs %zu bytes of shared memory",
           smem);
  void (*fn)(const PqArgs) = kcap == 32 ? pq_scan_kernel<32>
                             : kcap == 128 ? pq_scan_kernel<128>
                                           : pq_scan_kernel<256>;
  MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  {
    ScopedTiming tm("ivfpq_scan", st);
    fn<<<(unsigned)(nq * nprobe), kPqThreads, smem, st>>>(a);
    MF_LAUNCH_CHECK();
  }
  MF_TRY(launch_merge(pd, pl, nq, nprobe, k, k, distances, labels, st));
  if (list_ids) MF_TRY(launch_map_ids(list_ids, labels, nq * (int64_t)k, st));
  return MF_OK;
}

}  // extern "C"
