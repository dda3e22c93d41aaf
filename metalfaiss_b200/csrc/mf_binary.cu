// Hamming k-NN and range search over packed binary codes: the B200 form of
// BinaryFlatIndex (python/metalfaiss/index/binary_flat_index.py:12-140), whose
// search counts the coordinates where a query and a row differ (:79-86; the
// vectors are 0/1 per coordinate, python/metalfaiss/index/binary_index.py:36-60).
//
// A vector of d bits is stored as W = ceil(d / 32) 32-bit words: bit j of the
// vector is bit j % 32 of word j / 32, padding bits zero. The distance of a
// (query, row) pair is sum_w popc(q[w] ^ x[w]): integer work bound by the
// integer pipe, with each row read once per 32-query tile.
//
// Blocks of 256 threads take a (32-query tile, row split) item. Per 128-row
// tile every thread computes 16 (query, row) distances (its row's words in
// registers, the queries' words broadcast from shared memory) into a shared
// tile, then each warp offers its 4 queries' 128 candidates to their warp
// top-k lists (mf_topk.cuh). Keys rank by (distance, row), so ties go to the
// lower row, as a stable sort of the distances does. Range search runs the
// same tiles twice: a count per (query, split), an exclusive scan into lims
// and per-split offsets, and a fill that writes each query's rows in row order.
#include "mf_scan.cuh"
#include "mf_timing.cuh"
#include "mf_topk.cuh"

namespace mf {
namespace {

constexpr int kBinQT = 32;       // queries per item
constexpr int kBinTR = 128;      // rows per tile
constexpr int kBinThreads = 256;
constexpr int kBinMaxW = 32;     // d <= 1024 bits
constexpr int kBinMaxSplits = 1024;

struct BinArgs {
  const uint32_t* xq;  // (nq, W)
  const uint32_t* xb;  // (nb, W)
  int64_t nq, nb;
  int W, k, nqt, splits;
  int64_t rows_per_split;
  float* out_d;        // top-k: (nq, splits, k) partials, or (nq, k) when splits == 1
  int64_t* out_l;
  int radius;          // range: rows with distance <= radius
  int64_t* counts;     // range: (nq, splits) counts (count pass) / offsets (fill pass)
};

__global__ void binary_pack_kernel(const uint8_t* __restrict__ x, int64_t n, int d, int W,
                                   uint32_t* __restrict__ codes) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * W) return;
  const int64_t r = i / W;
  const int w = (int)(i - r * W);
  const uint8_t* row = x + r * d;
  uint32_t v = 0;
  for (int b = 0; b < 32; ++b) {
    const int j = 32 * w + b;
    if (j < d && row[j] != 0) v |= 1u << b;
  }
  codes[i] = v;
}

__global__ void binary_unpack_kernel(const uint32_t* __restrict__ codes, int64_t n, int d, int W,
                                     uint8_t* __restrict__ x) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * d) return;
  const int64_t r = i / d;
  const int j = (int)(i - r * d);
  x[i] = (uint8_t)((codes[r * W + j / 32] >> (j % 32)) & 1u);
}

// Distances of this thread's row against queries [qb, qb + 16) of the tile,
// written to dt (0xffff where the row is outside the split).
template <int WMAX>
__device__ __forceinline__ void binary_tile(const BinArgs& a, const uint32_t (*qs)[kBinMaxW],
                                            uint16_t (*dt)[kBinTR], int64_t r0, int64_t re) {
  const int t = threadIdx.x;
  const int rr = t & (kBinTR - 1);
  const int qb = (t / kBinTR) * (kBinQT * kBinTR / kBinThreads);
  const int64_t row = r0 + rr;
  const bool valid = row < re;
  uint32_t x[WMAX];
  const uint32_t* src = a.xb + (valid ? row : 0) * a.W;
#pragma unroll
  for (int w = 0; w < WMAX; ++w) x[w] = (valid && w < a.W) ? __ldg(src + w) : 0u;
#pragma unroll 4
  for (int i = 0; i < kBinQT * kBinTR / kBinThreads; ++i) {
    const int q = qb + i;
    int h = 0;
#pragma unroll
    for (int w = 0; w < WMAX; ++w) h += __popc(x[w] ^ qs[q][w]);
    dt[q][rr] = valid ? (uint16_t)h : (uint16_t)0xffff;
  }
}

__device__ __forceinline__ void load_query_tile(const BinArgs& a, int qt, uint32_t (*qs)[kBinMaxW]) {
  for (int i = threadIdx.x; i < kBinQT * kBinMaxW; i += kBinThreads) {
    const int q = i / kBinMaxW, w = i % kBinMaxW;
    const int64_t gq = (int64_t)qt * kBinQT + q;
    qs[q][w] = (gq < a.nq && w < a.W) ? a.xq[gq * a.W + w] : 0u;
  }
}

template <int WMAX, int KCAP>
__global__ void __launch_bounds__(kBinThreads)
    binary_topk_kernel(const BinArgs a) {
  __shared__ uint32_t qs[kBinQT][kBinMaxW];
  __shared__ uint16_t dt[kBinQT][kBinTR];
  extern __shared__ unsigned long long bin_smem[];
  unsigned long long* lists = bin_smem;                 // kBinQT x KCAP
  unsigned long long* bufs = bin_smem + kBinQT * KCAP;  // kBinQT x 32
  const int item = blockIdx.x;
  const int qt = item % a.nqt;
  const int s = item / a.nqt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rb = (int64_t)s * a.rows_per_split;
  const int64_t re = rb + a.rows_per_split < a.nb ? rb + a.rows_per_split : a.nb;
  load_query_tile(a, qt, qs);
  WarpTopK<KCAP> st[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int q = warp * 4 + j;
    st[j].init(lists + q * KCAP, bufs + q * 32, a.k, lane);
  }
  __syncthreads();
  for (int64_t r0 = rb; r0 < re; r0 += kBinTR) {
    binary_tile<WMAX>(a, qs, dt, r0, re);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = warp * 4 + j;
      unsigned long long key[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = lane + 32 * i;
        const uint16_t h = dt[q][c];
        key[i] = h == 0xffff ? kEmptyKey : make_key((float)h, (unsigned int)(r0 + c));
      }
      st[j].offer4(key, a.k, lane);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    st[j].flush(a.k, lane);
    const int64_t gq = (int64_t)qt * kBinQT + warp * 4 + j;
    if (gq >= a.nq) continue;
    const int64_t base = (a.splits > 1 ? (gq * a.splits + s) : gq) * a.k;
    for (int i = lane; i < a.k; i += 32) {
      const unsigned long long key = st[j].list[i];
      a.out_d[base + i] = key == kEmptyKey ? __int_as_float(0x7f800000) : key_dist(key);
      a.out_l[base + i] = key == kEmptyKey ? -1 : (int64_t)key_index(key);
    }
  }
}

// Range search: FILL = false counts each (query, split)'s rows within the
// radius into a.counts; FILL = true writes them (distance, row) from the
// per-(query, split) offsets in a.counts, in row order.
template <int WMAX, bool FILL>
__global__ void __launch_bounds__(kBinThreads)
    binary_range_kernel(const BinArgs a) {
  __shared__ uint32_t qs[kBinQT][kBinMaxW];
  __shared__ uint16_t dt[kBinQT][kBinTR];
  const int item = blockIdx.x;
  const int qt = item % a.nqt;
  const int s = item / a.nqt;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rb = (int64_t)s * a.rows_per_split;
  const int64_t re = rb + a.rows_per_split < a.nb ? rb + a.rows_per_split : a.nb;
  load_query_tile(a, qt, qs);
  int64_t run[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int64_t gq = (int64_t)qt * kBinQT + warp * 4 + j;
    if (FILL && gq < a.nq) run[j] = a.counts[gq * a.splits + s];
  }
  __syncthreads();
  for (int64_t r0 = rb; r0 < re; r0 += kBinTR) {
    binary_tile<WMAX>(a, qs, dt, r0, re);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = warp * 4 + j;
      // padding queries of the last tile count nothing and write nothing
      const bool live = (int64_t)qt * kBinQT + q < a.nq;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = lane + 32 * i;
        const uint16_t h = dt[q][c];
        const bool in = live && h != 0xffff && (int)h <= a.radius;
        const unsigned int m = __ballot_sync(0xffffffffu, in);
        if (FILL && in) {
          const int64_t pos = run[j] + __popc(m & lanemask_lt());
          a.out_d[pos] = (float)h;
          a.out_l[pos] = r0 + c;
        }
        run[j] += __popc(m);
      }
    }
    __syncthreads();
  }
  if (!FILL && lane == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gq = (int64_t)qt * kBinQT + warp * 4 + j;
      if (gq < a.nq) a.counts[gq * a.splits + s] = run[j];
    }
  }
}

// Per query: counts (nq, splits) -> exclusive offsets within the query, and
// the query's total into lims[q + 1].
__global__ void binary_split_scan_kernel(int64_t* counts, int64_t nq, int splits, int64_t* lims) {
  const int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  int64_t acc = 0;
  for (int s = 0; s < splits; ++s) {
    const int64_t c = counts[q * splits + s];
    counts[q * splits + s] = acc;
    acc += c;
  }
  lims[q + 1] = acc;
}

// lims[0] = 0, lims[1..nq] inclusive prefix sums (one block, chunks of 1024).
__global__ void binary_lims_scan_kernel(int64_t* lims, int64_t nq) {
  __shared__ int64_t part[1024];
  __shared__ int64_t carry;
  if (threadIdx.x == 0) {
    carry = 0;
    lims[0] = 0;
  }
  __syncthreads();
  for (int64_t b = 0; b < nq; b += 1024) {
    const int64_t i = b + threadIdx.x;
    int64_t v = i < nq ? lims[i + 1] : 0;
    part[threadIdx.x] = v;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {
      const int64_t add = threadIdx.x >= o ? part[threadIdx.x - o] : 0;
      __syncthreads();
      part[threadIdx.x] += add;
      __syncthreads();
    }
    if (i < nq) lims[i + 1] = part[threadIdx.x] + carry;
    __syncthreads();
    if (threadIdx.x == 1023) carry += part[1023];
    __syncthreads();
  }
}

// Per query: its split offsets shifted by lims[q].
__global__ void binary_offsets_kernel(int64_t* counts, int64_t nq, int splits,
                                      const int64_t* lims) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * splits) return;
  counts[i] += lims[i / splits];
}

// Binary IVF: one block per (query, probe) pair. The query's words sit in
// shared memory; the warps take the list's rows 32 at a time (one row per
// lane, rows `pitch` words apart), feed per-warp top-k lists, and warp 0
// merges them into the pair's k best. A candidate's index is
// (probe rank << 26) | (offset in its list), so the merge across probes orders
// ties by probe, then by row: the order in which the reference concatenates a
// query's candidates (python/metalfaiss/index/binary_ivf_index.py:150-175).
constexpr int kBinIvfOffBits = 26;

template <int WMAX, int KCAP>
__global__ void __launch_bounds__(kBinThreads)
    binary_ivf_kernel(const uint32_t* __restrict__ xq, int W, const int64_t* __restrict__ probes,
                      int P, int nlist, const int64_t* __restrict__ offsets,
                      const uint32_t* __restrict__ codes, int pitch, int k, float* out_d,
                      int64_t* out_l) {
  extern __shared__ unsigned long long bin_smem[];
  unsigned long long* lists = bin_smem;                         // 8 x KCAP
  unsigned long long* bufs = bin_smem + (kBinThreads / 32) * KCAP;  // 8 x 32
  __shared__ uint32_t qw[kBinMaxW];
  const int pair = blockIdx.x;
  const int64_t q = pair / P;
  const int pr = pair - (int)(q * P);
  const int64_t l = probes[pair];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* od = out_d + (size_t)pair * k;
  int64_t* ol = out_l + (size_t)pair * k;
  if (l < 0 || l >= nlist) {
    for (int i = threadIdx.x; i < k; i += kBinThreads) {
      od[i] = __int_as_float(0x7f800000);
      ol[i] = -1;
    }
    return;
  }
  if (threadIdx.x < kBinMaxW) qw[threadIdx.x] = threadIdx.x < W ? xq[q * W + threadIdx.x] : 0u;
  WarpTopK<KCAP> tk;
  tk.init(lists + warp * KCAP, bufs + warp * 32, k, lane);
  __syncthreads();
  uint32_t qr[WMAX];
#pragma unroll
  for (int w = 0; w < WMAX; ++w) qr[w] = qw[w];
  const int64_t rb = offsets[l];
  // rows past 2^26 of one list cannot be tagged; the entry point documents
  // the limit, and they are left out rather than mislabelled
  const int64_t re = offsets[l + 1] - rb > (1ll << kBinIvfOffBits) ? rb + (1ll << kBinIvfOffBits)
                                                                    : offsets[l + 1];
  const unsigned int tag = (unsigned int)pr << kBinIvfOffBits;
  for (int64_t r0 = rb + 32 * warp; r0 < re; r0 += kBinThreads) {
    const int64_t row = r0 + lane;
    unsigned long long key = kEmptyKey;
    if (row < re) {
      const uint32_t* c = codes + row * pitch;
      int h = 0;
#pragma unroll
      for (int w = 0; w < WMAX; ++w)
        if (w < W) h += __popc(c[w] ^ qr[w]);
      key = make_key((float)h, tag | (unsigned int)(row - rb));
    }
    tk.offer(key, k, lane);
  }
  tk.flush(k, lane);
  __syncthreads();
  if (warp == 0) {
    for (int w = 1; w < kBinThreads / 32; ++w)
      for (int i = 0; i < k; i += 32)
        tk.offer(i + lane < k ? lists[w * KCAP + i + lane] : kEmptyKey, k, lane);
    tk.flush(k, lane);
    for (int i = lane; i < k; i += 32) {
      const unsigned long long key = tk.list[i];
      od[i] = key == kEmptyKey ? __int_as_float(0x7f800000) : key_dist(key);
      ol[i] = key == kEmptyKey ? -1 : (int64_t)key_index(key);
    }
  }
}

// (probe rank << 26 | offset) -> ids[offsets[probes[q][rank]] + offset] (or
// the row position when ids is NULL); -1 stays.
__global__ void binary_ivf_labels_kernel(int64_t* labels, int64_t nq, int k, int P,
                                         const int64_t* __restrict__ probes,
                                         const int64_t* __restrict__ offsets,
                                         const int64_t* __restrict__ ids) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nq * k) return;
  const int64_t v = labels[i];
  if (v < 0) return;
  const int64_t q = i / k;
  const int pr = (int)(v >> kBinIvfOffBits);
  if (pr >= P) {
    labels[i] = -1;
    return;
  }
  const int64_t off = v & ((1ll << kBinIvfOffBits) - 1);
  const int64_t row = offsets[probes[q * P + pr]] + off;
  labels[i] = ids ? ids[row] : row;
}

// About two waves of blocks; every split at least one tile.
void binary_plan(int64_t nq, int64_t nb, int device, int* nqt, int* splits, int64_t* rps) {
  *nqt = (int)ceil_div(nq, kBinQT);
  const long long target = 2ll * (device >= 0 ? num_sms(device) : 148) * 4;
  long long s = ceil_div(target, *nqt > 0 ? *nqt : 1);
  const long long max_s = nb > 0 ? ceil_div(nb, kBinTR) : 1;
  if (s > max_s) s = max_s;
  if (s > kBinMaxSplits) s = kBinMaxSplits;
  if (s < 1) s = 1;
  long long r = ceil_div(nb > 0 ? nb : 1, s);
  r = ceil_div(r, kBinTR) * kBinTR;
  *splits = (int)ceil_div(nb > 0 ? nb : 1, r);
  *rps = r;
}

int bin_kcap(int k) { return k <= 32 ? 32 : (k <= 128 ? 128 : (k <= 256 ? 256 : 0)); }

template <int WMAX>
int launch_topk_w(const BinArgs& a, int kcap, int64_t items, cudaStream_t st) {
  const size_t smem = size_t(kBinQT) * (kcap + 32) * 8;
  void (*fn)(const BinArgs) = kcap == 32    ? binary_topk_kernel<WMAX, 32>
                              : kcap == 128 ? binary_topk_kernel<WMAX, 128>
                                            : binary_topk_kernel<WMAX, 256>;
  // the lists may pass the 48 KB a launch gets without asking
  MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  fn<<<(unsigned)items, kBinThreads, smem, st>>>(a);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

template <int WMAX>
int launch_range_w(const BinArgs& a, bool fill, int64_t items, cudaStream_t st) {
  if (fill)
    binary_range_kernel<WMAX, true><<<(unsigned)items, kBinThreads, 0, st>>>(a);
  else
    binary_range_kernel<WMAX, false><<<(unsigned)items, kBinThreads, 0, st>>>(a);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_topk(const BinArgs& a, int kcap, int64_t items, cudaStream_t st) {
  if (a.W <= 2) return launch_topk_w<2>(a, kcap, items, st);
  if (a.W <= 4) return launch_topk_w<4>(a, kcap, items, st);
  if (a.W <= 8) return launch_topk_w<8>(a, kcap, items, st);
  if (a.W <= 16) return launch_topk_w<16>(a, kcap, items, st);
  return launch_topk_w<32>(a, kcap, items, st);
}

template <int WMAX>
int launch_ivf_w(const uint32_t* xq, int W, const int64_t* probes, int P, int nlist,
                 const int64_t* offsets, const uint32_t* codes, int pitch, int k, int kcap,
                 float* pd, int64_t* pl, int64_t pairs, cudaStream_t st) {
  const size_t smem = size_t(kBinThreads / 32) * (kcap + 32) * 8;
  void (*fn)(const uint32_t*, int, const int64_t*, int, int, const int64_t*, const uint32_t*, int,
             int, float*, int64_t*) = kcap == 32    ? binary_ivf_kernel<WMAX, 32>
                                      : kcap == 128 ? binary_ivf_kernel<WMAX, 128>
                                                    : binary_ivf_kernel<WMAX, 256>;
  MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  fn<<<(unsigned)pairs, kBinThreads, smem, st>>>(xq, W, probes, P, nlist, offsets, codes, pitch, k,
                                                 pd, pl);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_ivf(const uint32_t* xq, int W, const int64_t* probes, int P, int nlist,
               const int64_t* offsets, const uint32_t* codes, int pitch, int k, float* pd,
               int64_t* pl, int64_t pairs, cudaStream_t st) {
  const int kcap = bin_kcap(k);
  if (W <= 2) return launch_ivf_w<2>(xq, W, probes, P, nlist, offsets, codes, pitch, k, kcap, pd, pl, pairs, st);
  if (W <= 4) return launch_ivf_w<4>(xq, W, probes, P, nlist, offsets, codes, pitch, k, kcap, pd, pl, pairs, st);
  if (W <= 8) return launch_ivf_w<8>(xq, W, probes, P, nlist, offsets, codes, pitch, k, kcap, pd, pl, pairs, st);
  if (W <= 16) return launch_ivf_w<16>(xq, W, probes, P, nlist, offsets, codes, pitch, k, kcap, pd, pl, pairs, st);
  return launch_ivf_w<32>(xq, W, probes, P, nlist, offsets, codes, pitch, k, kcap, pd, pl, pairs, st);
}

int launch_range(const BinArgs& a, bool fill, int64_t items, cudaStream_t st) {
  if (a.W <= 2) return launch_range_w<2>(a, fill, items, st);
  if (a.W <= 4) return launch_range_w<4>(a, fill, items, st);
  if (a.W <= 8) return launch_range_w<8>(a, fill, items, st);
  if (a.W <= 16) return launch_range_w<16>(a, fill, items, st);
  return launch_range_w<32>(a, fill, items, st);
}

int check_bin_shape(int64_t nq, int64_t nb, int d) {
  MF_CHECK(d > 0 && d % 8 == 0 && d <= 32 * kBinMaxW, MF_ERR_INVALID_ARGS,
           "binary dimension d=%d must be a multiple of 8 in [8, %d]", d, 32 * kBinMaxW);
  MF_CHECK(nq >= 0 && nb >= 0, MF_ERR_INVALID_ARGS, "negative sizes");
  MF_CHECK(nb < (1ll << 31) - 1, MF_ERR_INVALID_ARGS, "nb=%lld exceeds 2^31-2 rows per call",
           (long long)nb);
  return MF_OK;
}

size_t binary_ws_bytes(int64_t nq, int64_t nb, int k, int device) {
  int nqt, splits;
  int64_t rps;
  binary_plan(nq, nb, device, &nqt, &splits, &rps);
  Carver c(nullptr, 0);
  c.take<float>((size_t)nq * splits * (k > 0 ? k : 1));
  c.take<int64_t>((size_t)nq * splits * (k > 0 ? k : 1));
  c.take<int64_t>((size_t)nq * splits);
  return c.used;
}

}  // namespace
}  // namespace mf

using namespace mf;

#define MF_BIN_ENTER(device)                 \
  clear_error();                             \
  DeviceGuard _guard(device);                \
  if (_guard.status != MF_OK) return _guard.status

extern "C" {

int mf_binary_pack(int device, void* stream, const uint8_t* x, int64_t n, int d,
                   uint32_t* codes) {
  MF_BIN_ENTER(device);
  MF_TRY(check_bin_shape(0, n, d));
  if (n == 0) return MF_OK;
  MF_TRY(check_device_ptr(x, "x"));
  MF_TRY(check_device_ptr(codes, "codes"));
  const int W = (d + 31) / 32;
  const int64_t total = n * W;
  binary_pack_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, (cudaStream_t)stream>>>(x, n, d, W,
                                                                                      codes);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int mf_binary_unpack(int device, void* stream, const uint32_t* codes, int64_t n, int d,
                     uint8_t* x) {
  MF_BIN_ENTER(device);
  MF_TRY(check_bin_shape(0, n, d));
  if (n == 0) return MF_OK;
  MF_TRY(check_device_ptr(codes, "codes"));
  MF_TRY(check_device_ptr(x, "x"));
  const int W = (d + 31) / 32;
  binary_unpack_kernel<<<(unsigned)ceil_div(n * d, 256), 256, 0, (cudaStream_t)stream>>>(
      codes, n, d, W, x);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int mf_binary_flat_search_workspace_size(int64_t nq, int64_t nb, int d, int k, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_bin_shape(nq, nb, d));
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d must be in [1, %d]", k, kMaxK);
  int dev = 0;
  cudaGetDevice(&dev);
  *bytes = binary_ws_bytes(nq, nb, k, dev);
  return MF_OK;
}

int mf_binary_flat_search(int device, void* stream, const uint32_t* xq, int64_t nq,
                          const uint32_t* xb, int64_t nb, int d, int k, const int64_t* ids,
                          float* distances, int64_t* labels, void* workspace,
                          size_t workspace_bytes) {
  MF_BIN_ENTER(device);
  MF_TRY(check_bin_shape(nq, nb, d));
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d must be in [1, %d]", k, kMaxK);
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  MF_TRY(check_device_ptr(ids, "ids", true));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace", true));
  cudaStream_t st = (cudaStream_t)stream;
  BinArgs a{};
  a.xq = xq;
  a.xb = xb;
  a.nq = nq;
  a.nb = nb;
  a.W = (d + 31) / 32;
  a.k = k;
  binary_plan(nq, nb, device, &a.nqt, &a.splits, &a.rows_per_split);
  Carver c(workspace, workspace_bytes);
  float* pd = c.take<float>((size_t)nq * a.splits * k);
  int64_t* pl = c.take<int64_t>((size_t)nq * a.splits * k);
  c.take<int64_t>((size_t)nq * a.splits);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "binary search workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  a.out_d = a.splits > 1 ? pd : distances;
  a.out_l = a.splits > 1 ? pl : labels;
  const int64_t items = (int64_t)a.nqt * a.splits;
  {
    ScopedTiming tm("binary_topk", st);
    MF_TRY(launch_topk(a, bin_kcap(k), items, st));
  }
  if (a.splits > 1) MF_TRY(launch_merge(pd, pl, nq, a.splits, k, k, distances, labels, st));
  if (ids) MF_TRY(launch_map_ids(ids, labels, nq * (int64_t)k, st));
  return MF_OK;
}

int mf_binary_range_workspace_size(int64_t nq, int64_t nb, int d, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_bin_shape(nq, nb, d));
  int dev = 0;
  cudaGetDevice(&dev);
  int nqt, splits;
  int64_t rps;
  binary_plan(nq, nb, dev, &nqt, &splits, &rps);
  Carver c(nullptr, 0);
  c.take<int64_t>((size_t)nq * splits);
  *bytes = c.used;
  return MF_OK;
}

// Pass 1: lims (nq + 1) and *total; the workspace keeps the per-split offsets
// for pass 2 (mf_binary_range_fill, same arguments and workspace).
int mf_binary_range_count(int device, void* stream, const uint32_t* xq, int64_t nq,
                          const uint32_t* xb, int64_t nb, int d, int radius, int64_t* lims,
                          int64_t* total, void* workspace, size_t workspace_bytes) {
  MF_BIN_ENTER(device);
  MF_TRY(check_bin_shape(nq, nb, d));
  MF_CHECK(total != nullptr, MF_ERR_INVALID_ARGS, "total is NULL");
  *total = 0;
  MF_TRY(check_device_ptr(lims, "lims"));
  cudaStream_t st = (cudaStream_t)stream;
  if (nq == 0) {
    MF_CUDA(cudaMemsetAsync(lims, 0, sizeof(int64_t), st));
    return MF_OK;
  }
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  BinArgs a{};
  a.xq = xq;
  a.xb = xb;
  a.nq = nq;
  a.nb = nb;
  a.W = (d + 31) / 32;
  a.radius = radius;
  binary_plan(nq, nb, device, &a.nqt, &a.splits, &a.rows_per_split);
  Carver c(workspace, workspace_bytes);
  a.counts = c.take<int64_t>((size_t)nq * a.splits);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "binary range workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  MF_TRY(launch_range(a, false, (int64_t)a.nqt * a.splits, st));
  binary_split_scan_kernel<<<(unsigned)ceil_div(nq, 256), 256, 0, st>>>(a.counts, nq, a.splits,
                                                                         lims);
  MF_LAUNCH_CHECK();
  binary_lims_scan_kernel<<<1, 1024, 0, st>>>(lims, nq);
  MF_LAUNCH_CHECK();
  binary_offsets_kernel<<<(unsigned)ceil_div(nq * a.splits, 256), 256, 0, st>>>(a.counts, nq,
                                                                                a.splits, lims);
  MF_LAUNCH_CHECK();
  MF_CUDA(cudaMemcpyAsync(total, lims + nq, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  MF_CUDA(cudaStreamSynchronize(st));
  return MF_OK;
}

int mf_binary_range_fill(int device, void* stream, const uint32_t* xq, int64_t nq,
                         const uint32_t* xb, int64_t nb, int d, int radius,
                         const int64_t* lims, const int64_t* ids, float* distances,
                         int64_t* labels, void* workspace, size_t workspace_bytes) {
  MF_BIN_ENTER(device);
  MF_TRY(check_bin_shape(nq, nb, d));
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  MF_TRY(check_device_ptr(lims, "lims"));
  MF_TRY(check_device_ptr(ids, "ids", true));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  cudaStream_t st = (cudaStream_t)stream;
  BinArgs a{};
  a.xq = xq;
  a.xb = xb;
  a.nq = nq;
  a.nb = nb;
  a.W = (d + 31) / 32;
  a.radius = radius;
  a.out_d = distances;
  a.out_l = labels;
  binary_plan(nq, nb, device, &a.nqt, &a.splits, &a.rows_per_split);
  Carver c(workspace, workspace_bytes);
  a.counts = c.take<int64_t>((size_t)nq * a.splits);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "binary range workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  MF_TRY(launch_range(a, true, (int64_t)a.nqt * a.splits, st));
  int64_t total = 0;
  MF_CUDA(cudaMemcpyAsync(&total, lims + nq, sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  MF_CUDA(cudaStreamSynchronize(st));
  if (ids && total > 0) MF_TRY(launch_map_ids(ids, labels, total, st));
  return MF_OK;
}

int mf_binary_ivf_search_workspace_size(int64_t nq, int nprobe, int k, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_CHECK(k >= 1 && k <= kMaxK && nprobe >= 1 && nq >= 0, MF_ERR_INVALID_ARGS, "k=%d nprobe=%d",
           k, nprobe);
  Carver c(nullptr, 0);
  c.take<float>((size_t)nq * nprobe * k);
  c.take<int64_t>((size_t)nq * nprobe * k);
  *bytes = c.used;
  return MF_OK;
}

int mf_binary_ivf_search(int device, void* stream, const uint32_t* xq, int64_t nq,
                         const int64_t* probes, int nprobe, int nlist,
                         const int64_t* list_offsets, const uint32_t* list_codes, int code_pitch,
                         const int64_t* list_ids, int d, int k, float* distances,
                         int64_t* labels, void* workspace, size_t workspace_bytes) {
  MF_BIN_ENTER(device);
  MF_TRY(check_bin_shape(nq, 0, d));
  const int W = (d + 31) / 32;
  MF_CHECK(code_pitch >= W, MF_ERR_INVALID_ARGS, "code pitch %d < %d words", code_pitch, W);
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d must be in [1, %d]", k, kMaxK);
  MF_CHECK(nprobe >= 1 && nprobe <= 64 && nlist >= 1, MF_ERR_INVALID_ARGS,
           "nprobe=%d (1 to 64), nlist=%d", nprobe, nlist);
  MF_CHECK(nq * nprobe < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(probes, "probes"));
  MF_TRY(check_device_ptr(list_offsets, "list_offsets"));
  MF_TRY(check_device_ptr(list_codes, "list_codes", true));
  MF_TRY(check_device_ptr(list_ids, "list_ids", true));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  float* pd = c.take<float>((size_t)nq * nprobe * k);
  int64_t* pl = c.take<int64_t>((size_t)nq * nprobe * k);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "binary IVF workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  cudaStream_t st = (cudaStream_t)stream;
  {
    ScopedTiming tm("binary_ivf", st);
    MF_TRY(launch_ivf(xq, W, probes, nprobe, nlist, list_offsets, list_codes, code_pitch, k, pd, pl,
                      nq * nprobe, st));
  }
  MF_TRY(launch_merge(pd, pl, nq, nprobe, k, k, distances, labels, st));
  binary_ivf_labels_kernel<<<(unsigned)ceil_div(nq * k, 256), 256, 0, st>>>(
      labels, nq, k, nprobe, probes, list_offsets, list_ids);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

}  // extern "C"
