// IVF filter search (L2): an fp16 tensor-core pass (tq_scan_kernel with FLT,
// mf_tc.cu) keeps, per (query, probe) pair, up to `slots` smallest upper
// bounds on the rows' exact distances; this file builds the bank it reads,
// the per-pair scales and error bounds, and the exact fp32 refinement that
// follows. The results are those of the exact scan: the error bound below is
// rigorous, and a pair whose kept slots cannot prove that they hold every row
// that may belong to the top-k has its list rescanned exactly.
//
// Operands. Row x of list l (centroid c) is stored as fp16(s_l (x - c)) and
// the query as fp16(s_q (q - c)), rounded to nearest; s_l and s_q are powers
// of two that bring the list's largest residual norm R_l and |q - c| into
// [2^11, 2^12), so no element overflows and, short of elements below 2^-38 of
// those norms, none is subnormal. The tensor cores accumulate the products
// (exact in fp32) in fp32; 1 / (s_q s_l) scales the result back exactly.
//
// Error bound of a pair. The scan forms  a = Dc + rn_x - 2 <q', x'>~  with
// q' = q - c, x' = x - c, Dc = |q'|^2 and rn_x = |x'|^2 in fp32. Rounding an
// element to fp16 moves it by at most 2^-11 of itself (or 2^-25 / s in
// absolute terms where it underflows), so by Cauchy-Schwarz
//   |<q', x'> - <q', x'>~| <= (2^-10 + 2^-22 + acc (1 + 2^-10)) |q'| |x'| + underflow,
// where acc bounds the tensor cores' fp32 accumulation of the d exact
// products relative to the sum of their magnitudes. acc = d 2^-22 (2^-15 at
// d = 128): every addend truncated by less than one unit in the 24th
// significant bit of the largest term of its addition, however many terms the
// hardware adds at once. That covers the multi-term additions that align to
// the largest exponent and truncate, as published measurements describe NVIDIA
// tensor cores (Fasi, Higham, Mikaitis, Pranesh, "Numerical behavior of NVIDIA
// tensor cores", PeerJ Computer Science, 2021); round-to-nearest is tighter.
// mf_diag_f16_dot runs both instruction forms used here (tcgen05.mma kind::f16
// and mma.sync m16n8k16) so that tests measure this on the device with
// adversarial operands. With |q'| <= sqrt(Dc)(1 + 2^-17) and |x'| <= R_l
// (rounded up), and d <= 128, the pair's bound is
//   e = 2^-9 (1 + 2^-5 + 2^-9) sqrt(Dc) R_l                (the products)
//     + 2^-22 sqrt(d) (sqrt(Dc) / s_l + R_l / s_q)         (underflow)
//     + (d + 20) 2^-23 (|q|^2 + XN_l + Dc + R_l^2)         (fp32 rounding)
// where the last term covers the rounding of Dc, rn_x, the scan's own
// arithmetic and the refinement's distance t (each at most (d + 7) 2^-23
// times those magnitudes; XN_l is the list's largest |x|^2). So |a - t| <= e
// for every row of the list. A pair whose scales would leave fp32's range
// gets e = +inf: the scan keeps none of its rows and the refinement rescans
// its list exactly.
//
// The tensor-core pass folds rn_x into its accumulator: each bank row has a
// 16-element fp16 extension [hi, lo, 0, ...] with hi + lo = beta_l rn_x (beta_l
// a power of two per list bringing the list's largest rn_x under 2^15; lo the
// fp16 rounding of the remainder, so hi + lo is within 2^-22 of it), and each
// pair's query row the extension [A_e, A_e, 0, ...] with A_e = -s_q s_l /
// (2 beta_l), a power of two. The accumulator is then s_q s_l (<q', x'>~ - rn_x
// / 2), and u = (Dc + e) - 2 acc / (s_q s_l): one compare per column against a
// per-row constant decides the filter. The two extra products enter the
// accumulation bound, adding (d + 3) 2^-22 R_l^2 to e (the accumulation over
// d + 2 terms of magnitude up to s_q s_l R_l^2 / 2 each, and the hi/lo
// representation); a pair whose A_e is not an fp16 power of two gets
// e = +inf (its list is rescanned exactly).
//
// Selection. The scan keeps u = max(a + e, 0) >= t, with t >= u - 2e. Let B be
// the query's bound from the first rows of its nearest list (an upper bound
// on its k-th exact distance T_k) and U the k-th smallest u over its probes
// (U >= T_k, as u >= t row by row). A row of list l can be in the top-k only
// if t <= T_k <= W = min(U, B), hence only if u <= W + 2e. The scan keeps
// rows with u <= B + 2e (which is >= W + 2e) and of those the `slots`
// smallest u, so a pair's slots hold every row with u <= W + 2e unless they
// are all taken and the last one is <= W + 2e; that pair's list is then
// rescanned exactly. The refinement computes t for every kept row with
// u <= W + 2e (and every row of a rescanned list) and selects the top-k by
// (t, row), keeping only t <= W.
#include <cuda_fp16.h>

#include "mf_filter.cuh"
#include "mf_timing.cuh"
#include "mf_topk.cuh"

namespace mf {
namespace {

__device__ unsigned long long g_filter_rescans = 0;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ uint32_t f16x2_bits(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The power-of-two exponent that brings a norm n into [2^11, 2^12) (0 for 0).
__device__ __forceinline__ int scale_exp(float n) {
  if (!(n > 0.0f)) return 0;
  int e;
  frexpf(n, &e);  // n = m 2^e, 0.5 <= m < 1
  return 12 - e;
}

constexpr int kBankThreads = 256;
constexpr int kScaleExpMax = 60;  // |exponent| of a list's or a query's scale

// One block per list; warp w takes rows w, w + 8, ... of the list, lane j the
// elements [4j, 4j + 4) + 128 i of a row. First pass: the rows' squared
// residual norms and the list's largest; second pass: the scaled fp16 rows.
// Per row also the 16-element fp16 norm extension (two uint4 words) for the
// tensor-core pass: [hi, lo, 0, ...] of beta_l rn_x, and stats.w = beta_l.
__global__ void __launch_bounds__(kBankThreads) filter_bank_kernel(
    int d, const int64_t* __restrict__ offsets, const float* __restrict__ xb,
    const float* __restrict__ xnorms, const float* __restrict__ cents, uint2* h, float* rn,
    float4* stats, uint4* rn16) {
  const int l = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rb = offsets[l];
  const int64_t re = offsets[l + 1];
  const float* c = cents + (int64_t)l * d;
  float mr = 0.0f, mx = 0.0f;
  for (int64_t r = rb + warp; r < re; r += kBankThreads / 32) {
    const float* x = xb + r * d;
    float s = 0.0f;
    for (int j = 4 * lane; j < d; j += 128) {
      const float4 xv = *reinterpret_cast<const float4*>(x + j);
      const float4 cv = *reinterpret_cast<const float4*>(c + j);
      const float v0 = xv.x - cv.x, v1 = xv.y - cv.y, v2 = xv.z - cv.z, v3 = xv.w - cv.w;
      s = fmaf(v0, v0, s);
      s = fmaf(v1, v1, s);
      s = fmaf(v2, v2, s);
      s = fmaf(v3, v3, s);
    }
    s = warp_sum(s);
    if (lane == 0) rn[r] = s;
    mr = fmaxf(mr, s);
    mx = fmaxf(mx, xnorms[r]);
  }
  __shared__ float s_r[kBankThreads / 32], s_x[kBankThreads / 32];
  __shared__ float s_scale, s_beta;
  mr = warp_max(mr);
  mx = warp_max(mx);
  if (lane == 0) {
    s_r[warp] = mr;
    s_x[warp] = mx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kBankThreads / 32; ++w) {
      mr = fmaxf(mr, s_r[w]);
      mx = fmaxf(mx, s_x[w]);
    }
    // rounded up: the fp32 sum of squares is within d 2^-24 of itself
    const float R = sqrtf(mr) * (1.0f + 0x1p-10f);
    int e = scale_exp(R);
    e = e > kScaleExpMax ? kScaleExpMax : (e < -kScaleExpMax ? -kScaleExpMax : e);
    s_scale = ldexpf(1.0f, e);
    // beta: R^2 beta < 2^15 (R = m 2^er with 0.5 <= m < 1, so R^2 < 2^(2 er))
    int er = 0;
    if (R > 0.0f) frexpf(R, &er);
    int eb = 15 - 2 * er;
    eb = eb > 2 * kScaleExpMax ? 2 * kScaleExpMax : (eb < -2 * kScaleExpMax ? -2 * kScaleExpMax : eb);
    s_beta = ldexpf(1.0f, eb);
    stats[l] = make_float4(R, mx, s_scale, s_beta);
  }
  __syncthreads();
  const float sl = s_scale;
  const float beta = s_beta;
  for (int64_t r = rb + threadIdx.x; r < re; r += kBankThreads) {
    const float v = rn[r] * beta;
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    const __half2 hl = __halves2half2(hi, lo);
    rn16[2 * r] = make_uint4(*reinterpret_cast<const uint32_t*>(&hl), 0u, 0u, 0u);
    rn16[2 * r + 1] = make_uint4(0u, 0u, 0u, 0u);
  }
  for (int64_t r = rb + warp; r < re; r += kBankThreads / 32) {
    const float* x = xb + r * d;
    for (int j = 4 * lane; j < d; j += 128) {
      const float4 xv = *reinterpret_cast<const float4*>(x + j);
      const float4 cv = *reinterpret_cast<const float4*>(c + j);
      h[(r * d + j) >> 2] = make_uint2(f16x2_bits((xv.x - cv.x) * sl, (xv.y - cv.y) * sl),
                                       f16x2_bits((xv.z - cv.z) * sl, (xv.w - cv.w) * sl));
    }
  }
}

// One warp per query: its row stays in registers (lane j: elements 4j + 128 i)
// while the warp walks its probes; lane p then writes pair p's values.
constexpr int kPairsWarps = 8;

#ifndef MF_PAIRS_BATCH
#define MF_PAIRS_BATCH 4
#endif
// Probes of a query whose centroid rows one warp loads at a time.
constexpr int kPairsBatch = MF_PAIRS_BATCH;

__global__ void __launch_bounds__(kPairsWarps * 32) filter_pairs_kernel(
    const float* __restrict__ xq, const float* __restrict__ qnorms, int64_t nq, int P, int d,
    const int64_t* __restrict__ probes, const int64_t* __restrict__ offsets, int nlist,
    const float* __restrict__ cents, const float4* __restrict__ stats,
    const float* __restrict__ bound, FilterPairs fp) {
  const int64_t q = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (q >= nq) return;  // warp-uniform
  constexpr int kMaxSlices = 8;  // d <= 1024
  float4 xv[kMaxSlices];
#pragma unroll
  for (int i = 0; i < kMaxSlices; ++i) {
    const int j = 4 * lane + 128 * i;
    xv[i] = j < d ? *reinterpret_cast<const float4*>(xq + q * d + j)
                  : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float qn = qnorms[q];
  const float bq = bound[q];
  for (int p0 = 0; p0 < P; p0 += 32) {
    // lane j ends with pair p0 + j's squared distance to its centroid
    float my_dc = 0.0f;
    const int np = P - p0 < 32 ? P - p0 : 32;
    const int64_t my_l = lane < np ? probes[q * P + p0 + lane] : -1;
    const bool my_ok = my_l >= 0 && my_l < nlist && offsets[my_l + 1] > offsets[my_l];
    // kPairsBatch probes at a time, so their centroid loads overlap
    constexpr int kB = kPairsBatch;
    for (unsigned int m = __ballot_sync(0xffffffffu, my_ok); m != 0u;) {
      int jj[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        jj[b] = m ? __ffs(m) - 1 : -1;
        if (m) m &= m - 1u;
      }
      float dc[kB];
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        dc[b] = 0.0f;
        if (jj[b] < 0) continue;
        const int64_t l = __shfl_sync(0xffffffffu, my_l, jj[b]);
        const float* c = cents + l * d;
#pragma unroll
        for (int i = 0; i < kMaxSlices; ++i) {
          const int e = 4 * lane + 128 * i;
          if (e < d) {
            const float4 cv = *reinterpret_cast<const float4*>(c + e);
            const float v0 = xv[i].x - cv.x, v1 = xv[i].y - cv.y, v2 = xv[i].z - cv.z,
                        v3 = xv[i].w - cv.w;
            dc[b] = fmaf(v0, v0, dc[b]);
            dc[b] = fmaf(v1, v1, dc[b]);
            dc[b] = fmaf(v2, v2, dc[b]);
            dc[b] = fmaf(v3, v3, dc[b]);
          }
        }
      }
#pragma unroll
      for (int b = 0; b < kB; ++b) {
        if (jj[b] < 0) continue;
        const float t = warp_sum(dc[b]);
        if (lane == jj[b]) my_dc = t;
      }
    }
    if (lane >= np) continue;
    const int64_t s = q * P + p0 + lane;
    // no kept slots until the scan writes them (a pair it does not scan keeps none)
    fp.cnt[s] = 0;
    if (!my_ok) {
      fp.qn[s] = 0.0f;
      fp.thr[s] = 0.0f;
      fp.e[s] = 0.0f;
      fp.sq[s] = 1.0f;
      fp.sc[s] = 1.0f;
      fp.ae[s] = 0.0f;
      continue;
    }
    const float dc = my_dc;
    const float4 st = stats[my_l];
    const float R = st.x, XN = st.y, sl = st.z, beta = st.w;
    const float nrm = sqrtf(dc) * (1.0f + 0x1p-17f);
    const int eq = scale_exp(nrm);
    float e, sq = 1.0f, sc = 1.0f, thr, ae = 0.0f;
    // the norm fold's multiplier -s_q s_l / (2 beta): an fp16 power of two
    const float ae_mag = eq > kScaleExpMax || eq < -kScaleExpMax
                             ? 0.0f : ldexpf(sl * 0.5f / beta, eq);
    if (eq > kScaleExpMax || eq < -kScaleExpMax || !(R * sl < 0x1p13f) ||
        !(ae_mag >= 0x1p-24f && ae_mag <= 0x1p15f)) {
      // out of the scales' range: keep nothing, rescan exactly
      e = __int_as_float(0x7f800000);
      thr = -1.0f;
    } else {
      sq = ldexpf(1.0f, eq);
      sc = 1.0f / (sq * sl);  // exact: a power of two within range
      // 0x1.09p-9 = 2^-9 (1 + 9 / 256) >= 2 (2^-10 + 2^-22 + 128 2^-22 (1 + 2^-10))
      // (1 + 2^-17) = 2^-9 (1.0315...): the products term for d <= 128
      e = 0x1.09p-9f * nrm * R + 0x1p-22f * sqrtf((float)d) * (nrm / sl + R / sq) +
          (float)(d + 20) * 0x1p-23f * (qn + XN + dc + R * R) +
          (float)(d + 3) * 0x1p-22f * R * R + 0x1p-100f;
      ae = -ae_mag;
      thr = bq + 2.0f * e;  // +inf stays +inf
    }
    fp.qn[s] = dc + e;
    fp.e[s] = e;
    fp.thr[s] = thr;
    fp.sq[s] = sq;
    fp.sc[s] = sc;
    fp.ae[s] = ae;
  }
}

constexpr int kRefineWarps = 4;
constexpr int kSlots = 32;

// Exact distances of the rows of list l, rows [rb, re), offered to `ex`
// (16 rows per step: each load brings one row across the warp), except the
// rows already offered from the pair's slots (`kept`: one row per lane, -1
// for none).
__device__ __forceinline__ void refine_rescan(const RefineArgs& f, const float4 qv, float qn,
                                              int64_t rb, int64_t re, int64_t kept,
                                              WarpTopK<kSlots>& ex, int k, int lane) {
  const int d = f.d;
  for (int64_t r0 = rb; r0 < re; r0 += 16) {
    const int64_t off = kept - r0;
    const unsigned int skip =
        __reduce_or_sync(0xffffffffu, (kept >= 0 && off >= 0 && off < 16) ? 1u << off : 0u);
    float pp[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int64_t r = r0 + i;
      float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < re && 4 * lane < d) xv = *reinterpret_cast<const float4*>(f.xb + r * d + 4 * lane);
      float t = xv.x * qv.x;
      t = fmaf(xv.y, qv.y, t);
      t = fmaf(xv.z, qv.z, t);
      pp[i] = fmaf(xv.w, qv.w, t);
    }
    const float dot = warp_transpose_reduce16(pp, lane);
    const int64_t my = r0 + (lane >> 1);
    const bool ok = my < re && (lane & 1) == 0 && !((skip >> (lane >> 1)) & 1u);
    unsigned long long key = kEmptyKey;
    if (ok) key = make_key(l2_from_dot(qn, f.xnorms[my], dot), (unsigned int)my);
    ex.offer(key, k, lane);
  }
}

// One warp per query. (1) U from the first k slots of every pair. (2) Exact
// distances of every kept row with u <= W + 2e (a pair whose slots are all
// taken contributes all of them). (3) For such a full pair, a row it did not
// keep has u >= its last kept u_S, so t >= u_S - 2e: it is rescanned only if
// that can still reach the k-th exact distance found so far (which only falls
// as rows are added). Pairs out of the scales' range (e = +inf) are rescanned.
__global__ void __launch_bounds__(kRefineWarps * 32) filter_refine_kernel(const RefineArgs f) {
  __shared__ unsigned long long s_list[kRefineWarps][2][kSlots];
  __shared__ unsigned long long s_buf[kRefineWarps][2][32];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t q = (int64_t)blockIdx.x * kRefineWarps + warp;
  if (q >= f.nq) return;  // warp-uniform; the kernel has no block-wide barrier
  const int k = f.k;
  const int d = f.d;
  const int S = f.slots;
  const float inf = __int_as_float(0x7f800000);
  const float4 qv = 4 * lane < d ? *reinterpret_cast<const float4*>(f.xq + q * d + 4 * lane)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
  const float qn = f.qnorms[q];

  WarpTopK<kSlots> uk;
  uk.init(s_list[warp][0], s_buf[warp][0], k, lane);
  for (int p0 = 0; p0 < f.P; p0 += 32) {
    // lane j holds pair p0 + j's count
    const int nl = p0 + lane < f.P ? f.cnt[q * f.P + p0 + lane] : 0;
    for (unsigned int m = __ballot_sync(0xffffffffu, nl > 0); m != 0u; m &= m - 1u) {
      const int j = __ffs(m) - 1;
      const int64_t s = q * f.P + p0 + j;
      const int n = __shfl_sync(0xffffffffu, nl, j);
      unsigned long long key = kEmptyKey;
      if (lane < k && lane < n) key = make_key(f.pd[s * S + lane], (unsigned int)f.pl[s * S + lane]);
      uk.offer(key, k, lane);
    }
  }
  uk.flush(k, lane);
  __syncwarp();
  const unsigned long long ukey = s_list[warp][0][k - 1];
  const float U = ukey == kEmptyKey ? inf : key_dist(ukey);
  const float Wb = fminf(U, f.bound[q]);

  WarpTopK<kSlots> ex;
  ex.init(s_list[warp][1], s_buf[warp][1], k, lane, bound_key(Wb));
  for (int p0 = 0; p0 < f.P; p0 += 32) {
    const bool in = p0 + lane < f.P;
    const int64_t sl = q * f.P + p0 + lane;
    const int nl = in ? f.cnt[sl] : 0;
    const float el = in ? f.pair_e[sl] : 0.0f;
    const int64_t ll = in ? f.probes[sl] : -1;
    // pairs out of the scales' range: rescan
    for (unsigned int m = __ballot_sync(0xffffffffu, ll >= 0 && el == inf); m != 0u;
         m &= m - 1u) {
      const int j = __ffs(m) - 1;
      const int64_t l = __shfl_sync(0xffffffffu, ll, j);
      if (lane == 0) atomicAdd(&g_filter_rescans, 1ull);
      refine_rescan(f, qv, qn, f.offsets[l], f.offsets[l + 1], -1, ex, k, lane);
    }
    unsigned int full = 0u;  // pairs whose slots are all taken within W + 2e
    for (unsigned int m = __ballot_sync(0xffffffffu, nl > 0 && el != inf); m != 0u;
         m &= m - 1u) {
      const int j = __ffs(m) - 1;
      const int64_t s = q * f.P + p0 + j;
      const int n = __shfl_sync(0xffffffffu, nl, j);
      const float W = Wb + 2.0f * __shfl_sync(0xffffffffu, el, j);
      const float u = lane < n ? f.pd[s * S + lane] : inf;
      const int64_t row = lane < n ? f.pl[s * S + lane] : -1;
      if (n == S && __shfl_sync(0xffffffffu, u, S - 1) <= W) full |= 1u << j;
      const unsigned int c = __ballot_sync(0xffffffffu, row >= 0 && u <= W);
      float my_t = 0.0f;
      for (unsigned int b = c; b != 0u; b &= b - 1u) {
        const int i = __ffs(b) - 1;
        const int64_t r = __shfl_sync(0xffffffffu, row, i);
        float4 xv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (4 * lane < d) xv = *reinterpret_cast<const float4*>(f.xb + r * d + 4 * lane);
        float t = xv.x * qv.x;
        t = fmaf(xv.y, qv.y, t);
        t = fmaf(xv.z, qv.z, t);
        t = fmaf(xv.w, qv.w, t);
        const float dot = warp_sum(t);
        if (lane == i) my_t = l2_from_dot(qn, f.xnorms[r], dot);
      }
      ex.offer(((c >> lane) & 1u) ? make_key(my_t, (unsigned int)row) : kEmptyKey, k, lane);
    }
    if (full == 0u) continue;
    ex.flush(k, lane);
    __syncwarp();
    for (unsigned int m = full; m != 0u; m &= m - 1u) {
      const int j = __ffs(m) - 1;
      const int64_t s = q * f.P + p0 + j;
      const unsigned long long kth = s_list[warp][1][k - 1];
      const float tk = kth == kEmptyKey ? inf : key_dist(kth);
      const float uS = f.pd[s * S + S - 1];
      const float e = __shfl_sync(0xffffffffu, el, j);
      // the smallest exact distance a row it did not keep can have, rounded down
      const float lo = (uS - 2.0f * e) - 0x1p-22f * (uS + 2.0f * e);
      if (lo > tk) continue;
      if (lane == 0) atomicAdd(&g_filter_rescans, 1ull);
      const int64_t l = __shfl_sync(0xffffffffu, ll, j);
      // its S kept rows were all offered above (each u <= u_S <= W)
      const int64_t kept = lane < S ? f.pl[s * S + lane] : -1;
      refine_rescan(f, qv, qn, f.offsets[l], f.offsets[l + 1], kept, ex, k, lane);
      ex.flush(k, lane);
      __syncwarp();
    }
  }
  ex.flush(k, lane);
  __syncwarp();
  for (int j = lane; j < k; j += 32) {
    const unsigned long long key = s_list[warp][1][j];
    float dv = inf;
    int64_t lv = -1;
    if (key != kEmptyKey) {
      dv = key_dist(key);
      const unsigned int pos = key_index(key);
      lv = f.ids ? f.ids[pos] : (int64_t)pos;
    }
    f.D[q * k + j] = dv;
    f.I[q * k + j] = lv;
  }
}

}  // namespace

int filter_slots_for(int k) {
  const int s = 2 * k > 16 ? 2 * k : 16;
  return s < kSlots ? s : kSlots;
}

int launch_filter_bank(int nlist, int d, const int64_t* offsets, const float* xb,
                       const float* xnorms, const float* cents, void* h, float* rn, float* stats,
                       void* rn16, cudaStream_t stream) {
  MF_CHECK(d > 0 && d % 8 == 0, MF_ERR_INVALID_ARGS, "filter bank needs d a multiple of 8 (d=%d)",
           d);
  if (nlist <= 0) return MF_OK;
  filter_bank_kernel<<<(unsigned int)nlist, kBankThreads, 0, stream>>>(
      d, offsets, xb, xnorms, cents, reinterpret_cast<uint2*>(h), rn,
      reinterpret_cast<float4*>(stats), reinterpret_cast<uint4*>(rn16));
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_filter_pairs(const float* xq, const float* qnorms, int64_t nq, int P, int d,
                        const int64_t* probes, const int64_t* offsets, int nlist,
                        const float* cents, const float* stats, const float* bound,
                        const FilterPairs& fp, cudaStream_t stream) {
  if (nq <= 0 || P <= 0) return MF_OK;
  MF_CHECK(d <= 1024, MF_ERR_INVALID_ARGS, "filter pairs: d=%d", d);
  ScopedTiming tm("ivf_filter_pairs", stream);
  filter_pairs_kernel<<<(unsigned int)ceil_div(nq, kPairsWarps), kPairsWarps * 32, 0, stream>>>(
      xq, qnorms, nq, P, d, probes, offsets, nlist, cents, reinterpret_cast<const float4*>(stats),
      bound, fp);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_filter_refine(const RefineArgs& f, cudaStream_t stream) {
  MF_CHECK(f.d <= 128 && f.d % 4 == 0 && f.k >= 1 && f.k <= f.slots && f.slots <= kSlots,
           MF_ERR_INVALID_ARGS, "filter refinement: d=%d k=%d slots=%d", f.d, f.k, f.slots);
  if (f.nq <= 0) return MF_OK;
  ScopedTiming tm("ivf_filter_refine", stream);
  filter_refine_kernel<<<(unsigned int)ceil_div(f.nq, kRefineWarps), kRefineWarps * 32, 0,
                         stream>>>(f);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int read_filter_rescans(unsigned long long* out, bool reset) {
  MF_CUDA(cudaMemcpyFromSymbol(out, g_filter_rescans, sizeof(unsigned long long)));
  if (reset) {
    const unsigned long long z = 0;
    MF_CUDA(cudaMemcpyToSymbol(g_filter_rescans, &z, sizeof(z)));
  }
  return MF_OK;
}

}  // namespace mf
