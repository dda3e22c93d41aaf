// Tensor-core slab scan (sm_100a): the L2 / inner-product distance tile of a
// work item (<= 32 queries x a slab of rows) computed by tcgen05 MMAs in
// 3xTF32 form with the accumulator in TMEM, fed to the same per-query warp
// top-k as the SIMT scan. Work items and outputs are exactly those of
// scan_kernel (mf_scan.cu), so either engine serves flat and IVF search.
//
// Per CTA (128 threads, one CTA per SM, persistent over work items):
//  * queries: gathered once per item, split into tf32 hi/lo and written as the
//    K-major B operand (N = 32 rows of 128-byte swizzled K-blocks);
//  * rows: 128-row x 32-float boxes stream in by TMA (128B swizzle, no
//    multicast) through a ring of SA stages, one stage per K-block;
//  * every stage is split in place (hi) plus a lo copy, then one thread issues
//    12 MMAs (4 K-steps x {hi.hi, hi.lo, lo.hi}) into one of two TMEM
//    accumulators (128 lanes x 32 columns each);
//  * the epilogue of tile t-1 (TMEM -> registers -> distances -> transposed
//    shared tile -> warp top-k) runs while tile t's MMAs execute.
// x.q = xh.qh + xh.ql + xl.qh, dropping xl.ql (relative size ~2^-22).
#include <cudaTypedefs.h>

#include <mutex>

#include "mf_scan.cuh"
#include "mf_sm100.cuh"
#include "mf_timing.cuh"
#include "mf_topk.cuh"

namespace mf {
namespace {
// Set by a kernel whose bounded wait gave up; read (and cleared) by
// mf_device_error(). Never set on the normal path.
__device__ int g_device_error = 0;
}  // namespace

namespace {
using namespace sm100;

#ifdef MF_TC_PROFILE
// Phase cycle counters of the tensor-core scan (instrumented builds only).
__device__ unsigned long long g_tc_prof[16];
#define TCP_DECL unsigned long long _tcp[16] = {0}; long long _tc0 = 0;
#define TCP_BEGIN() _tc0 = clock64()
#define TCP_END(i) _tcp[i] += (unsigned long long)(clock64() - _tc0)
#define TCP_FLUSH()                                                                  \
  if (tid == 0 || tid == 64)                                                         \
    for (int _i = 0; _i < 16; ++_i) atomicAdd(&g_tc_prof[_i], _tcp[_i]);
#else
#define TCP_DECL
#define TCP_BEGIN()
#define TCP_END(i)
#define TCP_FLUSH()
#endif

constexpr int kTcThreads = 256;
constexpr int kTcM = 128;                 // rows per tile (TMEM lanes)
constexpr int kTcN = 32;                  // queries per item (accumulator columns)
constexpr int kTcStageBytes = kTcM * 128;  // one 128 x 32 fp32 box
constexpr int kTcBBlockBytes = kTcN * 128;
constexpr int kTcMaxD = 256;
constexpr int kTcMaxSmem = 227 * 1024 - 256;  // dynamic part; static smem takes the rest

struct TcSmem {
  int SA;  // A stages
  int KB;  // K-blocks
  size_t a, l, bh, bl, t, lists, bufs, qout, qrow, qn, bars, total;
};

TcSmem tc_layout(int d, int kcap, int SA) {
  TcSmem s;
  s.SA = SA;
  s.KB = (d + 31) / 32;
  size_t o = 0;
  s.a = o;
  o += size_t(SA) * kTcStageBytes;
  s.l = o;
  o += size_t(2) * kTcStageBytes;
  s.bh = o;
  o += size_t(s.KB) * kTcBBlockBytes;
  s.bl = o;
  o += size_t(s.KB) * kTcBBlockBytes;
  s.t = o;
  o += size_t(kTcN) * kTcM * 4;
  s.lists = o;
  o += size_t(kTcN) * kcap * 8;
  s.bufs = o;
  o += size_t(kTcN) * 32 * 8;
  s.qout = o;
  o += kTcN * 8;
  s.qrow = o;
  o += kTcN * 4;
  s.qn = o;
  o += kTcN * 4;
  s.bars = o;
  o += size_t(2 * SA + 2) * 8 + 16;
  s.total = o + 1024;  // slack to align the base to 1024 bytes
  return s;
}

template <int METRIC, int KCAP>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_scan_kernel(const ScanArgs a, const __grid_constant__ CUtensorMap tmap, const TcSmem L) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* A = reinterpret_cast<float*>(base + L.a);
  float* Lo = reinterpret_cast<float*>(base + L.l);
  float* Bh = reinterpret_cast<float*>(base + L.bh);
  float* Bl = reinterpret_cast<float*>(base + L.bl);
  float* T = reinterpret_cast<float*>(base + L.t);
  unsigned long long* lists = reinterpret_cast<unsigned long long*>(base + L.lists);
  unsigned long long* bufs = reinterpret_cast<unsigned long long*>(base + L.bufs);
  long long* s_qout = reinterpret_cast<long long*>(base + L.qout);
  int* s_qrow = reinterpret_cast<int*>(base + L.qrow);
  float* s_qn = reinterpret_cast<float*>(base + L.qn);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
  uint64_t* mdone = full + L.SA;
  uint64_t* accf = mdone + L.SA;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accf + 2);
  int* s_abort = reinterpret_cast<int*>(s_tmem + 1);

  __shared__ int s_item;
  __shared__ long long s_rb, s_re;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int quad = warp & 3;   // TMEM lane quadrant this warp may access
  const int half = warp >> 2;  // which 16 of the 32 query columns it reads
  const int d = a.d;
  const int k = a.k;
  const int SA = L.SA;
  const int KB = L.KB;

  if (warp == 0) {
    tmem_alloc(s_tmem, 64);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&mdone[i], 1);
    }
    mbar_init(&accf[0], 1);
    mbar_init(&accf[1], 1);
    *s_abort = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  constexpr uint32_t idesc = idesc_tf32(kTcM, kTcN);

  TCP_DECL
#ifdef MF_TC_PROFILE
  const long long _t_start = clock64();
#endif
  uint32_t g = 0;         // A-stage sequence consumed so far (same in every thread)
  uint32_t g_issued = 0;  // A-stage sequence issued (thread 0)
  uint32_t tt = 0;        // tiles so far
  int next_load = 0;      // next K-block of the current item to load (thread 0)

  // Thread 0: issues the loads of the current item below `upto`; when `block`
  // is false it stops at the first stage whose previous MMAs are still running.
  auto pump = [&](int upto, bool block, long long rb, int nL) {
    if (upto > nL) upto = nL;
    while (next_load < upto) {
      const uint32_t seq = g + next_load;
      const int s = seq % SA;
      if (seq >= (uint32_t)SA) {
        const uint32_t par = ((seq / SA) - 1) & 1;
        if (block) mbar_wait(&mdone[s], par, s_abort, &g_device_error);
        else if (!mbar_test(&mdone[s], par)) break;
      }
      const int t = next_load / KB;
      const int kb = next_load - t * KB;
      mbar_arrive_expect_tx(&full[s], kTcStageBytes);
      tma_load_2d(A + size_t(s) * (kTcStageBytes / 4), &tmap, kb * 32,
                  (int)(rb + (long long)t * kTcM), &full[s]);
      g_issued = seq + 1;
      ++next_load;
    }
  };

  for (;;) {
    TCP_BEGIN();
    if (tid == 0) s_item = atomicAdd(a.counter, 1);
    __syncthreads();
    const int item = s_item;
    const int total = a.flat ? a.nqt * a.P : *a.item_total;
    if (item >= total || *s_abort) break;

    // ---- the work item: queries, output slots, row slab (as scan_kernel)
    if (a.flat) {
      const int qt = item % a.nqt;
      const int s = item / a.nqt;
      if (tid < kTcN) {
        long long q = (long long)qt * kTcN + tid;
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
      const int pb = a.pair_offsets[it.x] + it.y * kTcN;
      const int pe0 = a.pair_offsets[it.x + 1];
      const int pe = pe0 < pb + kTcN ? pe0 : pb + kTcN;
      if (tid < kTcN) {
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
        s_re = a.list_offsets[it.x + 1];
      }
    }
    __syncthreads();
    const long long rb = s_rb;
    const long long re = s_re;
    const long long nrows = re > rb ? re - rb : 0;
    const int nT = (int)((nrows + kTcM - 1) / kTcM);
    const int nL = nT * KB;
    if (tid == 0) {
      next_load = 0;
      pump(SA, false, rb, nL);  // start streaming rows while the queries are prepared
    }
    if (tid < kTcN) {
      const int qr = s_qrow[tid];
      s_qn[tid] = (METRIC == MF_METRIC_L2 && qr >= 0) ? a.qnorms[qr] : 0.0f;
    }
    // queries -> B operand (hi / lo), K-major, 128-byte swizzle
    for (int e = tid; e < kTcN * KB * 8; e += kTcThreads) {
      const int n = e / (KB * 8);
      const int rem = e - n * KB * 8;
      const int kb = rem >> 3;
      const int c = rem & 7;
      const int qr = s_qrow[n];
      const int col = kb * 32 + c * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (qr >= 0 && col < d) v = *reinterpret_cast<const float4*>(a.xq + (long long)qr * d + col);
      float4 h, l;
      split_tf32(v.x, h.x, l.x);
      split_tf32(v.y, h.y, l.y);
      split_tf32(v.z, h.z, l.z);
      split_tf32(v.w, h.w, l.w);
      const int off = kb * (kTcN * 32) + n * 32 + ((c ^ (n & 7)) << 2);
      *reinterpret_cast<float4*>(Bh + off) = h;
      *reinterpret_cast<float4*>(Bl + off) = l;
    }
    WarpTopK<KCAP> tk[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = warp * 4 + jj;
      tk[jj].init(lists + j * KCAP, bufs + j * 32, k, lane);
    }
    fence_proxy_async_smem();
    __syncthreads();
    TCP_END(0);

    // Epilogue of local tile u: accumulator -> distances -> top-k offers.
    auto epilogue = [&](int u) {
      const uint32_t ts = tt + u;
      const int b = ts & 1;
      TCP_BEGIN();
      mbar_wait(&accf[b], (ts >> 1) & 1, s_abort, &g_device_error);
      TCP_END(1);
      TCP_BEGIN();
      tc_fence_after();
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(quad * 32) << 16) + b * kTcN + half * 16, v);
      tc_fence_before();
      const long long r0 = rb + (long long)u * kTcM;
      const long long row = r0 + quad * 32 + lane;
      const bool valid = row < re;
      const float xn = (METRIC == MF_METRIC_L2 && valid) ? a.xnorms[row] : 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int j = half * 16 + i;
        float dist;
        if (METRIC == MF_METRIC_L2) dist = l2_from_dot(s_qn[j], xn, v[i]);
        else dist = -v[i];
        T[j * kTcM + quad * 32 + lane] = dist;
      }
      __syncthreads();
      TCP_END(2);
      TCP_BEGIN();
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int j = warp * 4 + jj;
        if (s_qrow[j] < 0) continue;
        unsigned long long key[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ri = i * 32 + lane;
          const long long r = r0 + ri;
          key[i] = r < re ? make_key(T[j * kTcM + ri], (unsigned int)r) : kEmptyKey;
        }
        tk[jj].offer4(key, k, lane);
      }
      TCP_END(3);
      TCP_BEGIN();
      __syncthreads();
      TCP_END(4);
    };

    for (int li = 0; li < nL; ++li) {
      const uint32_t seq = g + li;
      const int s = seq % SA;
      const int t = li / KB;
      const int kb = li - t * KB;
      const int lb = seq & 1;  // lo buffer
      TCP_BEGIN();
      if (tid == 0) pump(li + 1, true, rb, nL);  // this K-block's load must be in flight
      // the lo buffer was last read by the MMAs of sequence seq-2
      if (seq >= 2) mbar_wait(&mdone[(seq - 2) % SA], ((seq - 2) / SA) & 1, s_abort, &g_device_error);
      TCP_END(5);
      TCP_BEGIN();
      mbar_wait(&full[s], (seq / SA) & 1, s_abort, &g_device_error);
      TCP_END(6);
      TCP_BEGIN();
      float4* As = reinterpret_cast<float4*>(A + size_t(s) * (kTcStageBytes / 4));
      float4* Ls = reinterpret_cast<float4*>(Lo + size_t(lb) * (kTcStageBytes / 4));
#pragma unroll
      for (int e = tid; e < kTcStageBytes / 16; e += kTcThreads) {
        const float4 v = As[e];
        float4 h, l;
        split_tf32(v.x, h.x, l.x);
        split_tf32(v.y, h.y, l.y);
        split_tf32(v.z, h.z, l.z);
        split_tf32(v.w, h.w, l.w);
        As[e] = h;
        Ls[e] = l;
      }
      TCP_END(7);
      TCP_BEGIN();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      TCP_END(8);
      TCP_BEGIN();
      if (tid == 0) {
        const uint32_t dt = tmem + ((tt + t) & 1) * kTcN;
        const uint32_t a_addr = smem_u32(As);
        const uint32_t l_addr = smem_u32(Ls);
        const uint32_t bh_addr = smem_u32(Bh + kb * (kTcN * 32));
        const uint32_t bl_addr = smem_u32(Bl + kb * (kTcN * 32));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t off = kk * 32;  // 8 tf32 of K per MMA
          mma_tf32(dt, desc_k_sw128(a_addr + off), desc_k_sw128(bh_addr + off), idesc,
                   !(kb == 0 && kk == 0));
          mma_tf32(dt, desc_k_sw128(a_addr + off), desc_k_sw128(bl_addr + off), idesc, true);
          mma_tf32(dt, desc_k_sw128(l_addr + off), desc_k_sw128(bh_addr + off), idesc, true);
        }
        mma_commit(&mdone[s]);
        if (kb == KB - 1) mma_commit(&accf[(tt + t) & 1]);
        TCP_END(9);
        TCP_BEGIN();
        pump(li + SA, false, rb, nL);
        TCP_END(10);
      }
      if (kb == KB - 1 && t >= 1) epilogue(t - 1);
    }
    if (nT >= 1) epilogue(nT - 1);

    // ---- results of the item
    TCP_BEGIN();
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = warp * 4 + jj;
      if (s_qrow[j] < 0) continue;
      tk[jj].flush(k, lane);
      const long long slot = s_qout[j];
      for (int t = lane; t < k; t += 32) {
        const unsigned long long key = tk[jj].list[t];
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
    }
    g += nL;
    tt += nT;
    __syncthreads();
    TCP_END(11);
  }

#ifdef MF_TC_PROFILE
  _tcp[13] = (unsigned long long)(clock64() - _t_start);
  _tcp[14] = tt;
  _tcp[15] = g;
#endif
  TCP_FLUSH();
  // ---- teardown: copies and MMAs in flight finish before TMEM is released
  if (tid == 0) {
    int dummy = 0;
    for (uint32_t seq = g; seq < g_issued; ++seq)
      mbar_wait(&full[seq % SA], (seq / SA) & 1, &dummy, &g_device_error);
    if (g > 0) {
      dummy = 0;
      mbar_wait(&mdone[(g - 1) % SA], ((g - 1) / SA) & 1, &dummy, &g_device_error);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// ------------------------------------------------------------------ host
typedef void (*TcFn)(const ScanArgs, const CUtensorMap, const TcSmem);

template <int METRIC>
TcFn pick_tc(int kcap) {
  switch (kcap) {
    case 32: return tc_scan_kernel<METRIC, 32>;
    case 64: return tc_scan_kernel<METRIC, 64>;
    case 128: return tc_scan_kernel<METRIC, 128>;
    case 256: return tc_scan_kernel<METRIC, 256>;
  }
  return nullptr;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_tc_mu;
int g_tc_attr[64][2][4];  // smem limit set per (device, metric, kcap)

int encoder(PFN_cuTensorMapEncodeTiled_v12000* out) {
  std::lock_guard<std::mutex> lk(g_tc_mu);
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(MF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  *out = g_encode;
  return MF_OK;
}

int g_engine = 0;  // 0 auto, 1 SIMT only, 2 tensor cores where eligible

}  // namespace

void set_scan_engine(int e) { g_engine = e; }
int scan_engine() { return g_engine; }

bool tc_eligible(int metric, int d, int k, int64_t xb_rows) {
  if (g_engine != 2) return false;  // automatic selection keeps the SIMT scan for now
  if (metric != MF_METRIC_L2 && metric != MF_METRIC_INNER_PRODUCT) return false;
  if (d < 32 || d > kTcMaxD) return false;
  if (xb_rows < kTcM) return false;
  const int kcap = scan_kcap(k);
  if (kcap == 0) return false;
  return tc_layout(d, kcap, 2).total <= (size_t)kTcMaxSmem;
}

int launch_tc_scan(const ScanArgs& a, int metric, int64_t total_items, int64_t xb_rows,
                   int device, cudaStream_t stream) {
  const int kcap = scan_kcap(a.k);
  MF_CHECK(kcap != 0, MF_ERR_INVALID_ARGS, "k=%d exceeds %d", a.k, kMaxK);
  TcFn fn = metric == MF_METRIC_L2 ? pick_tc<MF_METRIC_L2>(kcap)
                                   : pick_tc<MF_METRIC_INNER_PRODUCT>(kcap);
  MF_CHECK(fn != nullptr, MF_ERR_METRIC, "metric %d has no tensor-core scan", metric);
  int SA = 8;
  TcSmem lay = tc_layout(a.d, kcap, SA);
  while (SA > 2 && lay.total > (size_t)kTcMaxSmem) lay = tc_layout(a.d, kcap, --SA);
  MF_CHECK(lay.total <= (size_t)kTcMaxSmem, MF_ERR_INVALID_ARGS,
           "tensor-core scan does not fit shared memory (d=%d k=%d)", a.d, a.k);
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  MF_TRY(encoder(&enc));
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)a.d, (cuuint64_t)xb_rows};
  cuuint64_t strides[1] = {(cuuint64_t)a.d * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)kTcM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.xb), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MF_CHECK(r == CUDA_SUCCESS, MF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    const int mi = metric == MF_METRIC_L2 ? 0 : 1;
    const int ki = kcap == 32 ? 0 : kcap == 64 ? 1 : kcap == 128 ? 2 : 3;
    if (device < 0 || device >= 64 || g_tc_attr[device][mi][ki] < (int)lay.total) {
      MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.total));
      if (device >= 0 && device < 64) g_tc_attr[device][mi][ki] = (int)lay.total;
    }
  }
  if (total_items <= 0) return MF_OK;
  long long grid = num_sms(device);
  if (grid > total_items) grid = total_items;
  MF_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(int), stream));
  ScopedTiming tm(a.flat ? "scan_topk_flat" : "scan_topk_ivf", stream);
  fn<<<(unsigned int)grid, kTcThreads, lay.total, stream>>>(a, map, lay);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

#ifdef MF_TC_PROFILE
extern "C" MF_API int mf_tc_profile_read(unsigned long long* out16, int reset) {
  MF_CUDA(cudaMemcpyFromSymbol(out16, g_tc_prof, 16 * sizeof(unsigned long long)));
  if (reset) {
    unsigned long long z[16] = {0};
    MF_CUDA(cudaMemcpyToSymbol(g_tc_prof, z, sizeof(z)));
  }
  return MF_OK;
}
#endif

int read_device_error(int* code) {
  int v = 0;
  MF_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  const int zero = 0;
  MF_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  *code = v;
  return MF_OK;
}

}  // namespace mf
