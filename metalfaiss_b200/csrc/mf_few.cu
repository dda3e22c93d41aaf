// Scan of IVF items that hold few queries (a list's last group of at most
// kFewMax queries): one block of four warps per item (two warps for items of
// at most kFewBoundRows rows, such as the bound pass's), the warps taking
// interleaved 16-row steps of the list, each with its own per-query top-k
// lists, merged at the end of the item. The item's queries sit in shared
// memory. Rows are read 16 at a time with
// fully coalesced loads (one load instruction = one whole row across the warp:
// lane l holds the row's 16-byte column slice l), each lane forms the partial
// dot products of its slice with every query, and a butterfly transpose-
// reduction (16 shuffles per query) leaves row i's sum in lanes 2i and 2i+1.
// These items hold most of a batch's probed rows but few (query, row) pairs,
// so the pass is bound by reading the rows once from HBM. Distances, keys and
// the per-query warp top-k are those of scan_kernel (mf_scan.cu), filtered by
// the per-query bound when one is given.
//
// FLT (L2, the filter search): the rows are the filter bank's fp16 residuals
// against the item's list centroid (scaled by the list's power of two), the
// queries s_q (q - c) rounded to fp16, and the dot products come from the
// tensor cores (mma.sync m16n8k16 with fp32 accumulation: 16 queries x 8 rows
// per instruction), the arithmetic of the tcgen05 filter pass, so the pair's
// error bound covers them. Each pair's keys are the filter's upper bounds
// u = (Dc + e) + rn_x - 2 dot, with the pair's query norm, bound and scales
// from a.pair_qn / pair_thr / pair_sc. A lane tests its 8 (query, row) bounds
// against the thresholds; only queries with a candidate gather their 16 rows'
// bounds to one lane each and take the per-query insertion above.
#include <cuda_fp16.h>

#include "mf_scan.cuh"
#include "mf_timing.cuh"
#include "mf_topk.cuh"

namespace mf {
namespace {

constexpr int kFewMax = 16;     // queries per item at most
#ifndef MF_FEW_WARPS
#define MF_FEW_WARPS 4
#endif
#ifndef MF_FEW_BOUND_WARPS
#define MF_FEW_BOUND_WARPS 2
#endif
constexpr int kFewWarps = MF_FEW_WARPS;  // warps per block, sharing one item (general items)
constexpr int kFewBoundWarps = MF_FEW_BOUND_WARPS;  // the same for the bound pass's items
constexpr int kFewBoundRows = 256;  // items of at most this many rows: kFewBoundWarps each
constexpr int kFewMaxD = 128;   // d at most: one 16-byte column slice per lane
constexpr int kFewK = 32;       // list slots per query (k <= 32)
constexpr int kFewRows = 16;    // rows per step

// Dynamic shared memory of a block of `warps` warps: the item's queries, then
// per warp the query lists (kFewK keys) and candidate buffers (32 keys).
struct FewSmem {
  __host__ __device__ static size_t queries(int d) { return size_t(kFewMax) * d * 4; }
  __host__ __device__ static size_t block(int d, int warps) {
    return queries(d) + size_t(warps) * kFewMax * (kFewK + 32) * 8;
  }
};

__device__ __forceinline__ uint32_t few_pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// c += A B for one m16n8k16 step: A 16 x 16 fp16 (four f16x2 registers per
// lane), B 16 x 8 fp16 (two), C 16 x 8 fp32
__device__ __forceinline__ void few_mma_f16(float (&c)[4], const uint32_t (&af)[4], uint32_t b0,
                                            uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(af[0]), "r"(af[1]), "r"(af[2]), "r"(af[3]), "r"(b0), "r"(b1));
}

// W warps per block share an item: 4 for general items (2 measured the same, 8
// a third slower: its block barriers wait on more warps); 2 for items of at
// most kFewBoundRows rows (the bound pass's 128: four steps each, 1-2 % faster
// than one warp at 10,000 queries and 8 % at 1,250). The fp16 form is held to
// 128 registers (16 warps per SM, no spills), so that each warp has two
// 16-row steps of loads in flight.
template <int METRIC, bool FLT, int W>
__global__ void __launch_bounds__(W * 32, FLT ? (W < 16 ? 16 / W : 1) : 1)
    few_scan_kernel(const ScanArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int d = a.d;
  const int k = a.k;
  const int d4 = d >> 2;
  float4* qs = reinterpret_cast<float4*>(smem_raw);  // kFewMax x d
  unsigned long long* lists_all =
      reinterpret_cast<unsigned long long*>(smem_raw + FewSmem::queries(d));
  unsigned long long* lists = lists_all + warp * kFewMax * (kFewK + 32);  // this warp's
  unsigned long long* bufs = lists + kFewMax * kFewK;
  __shared__ int s_item;
  __shared__ long long s_slot[kFewMax];
  __shared__ float s_qn[kFewMax];
  __shared__ float s_sc[kFewMax];
  __shared__ unsigned long long s_bnd[kFewMax];
  const int total = *a.item_total;
  const int group = a.group > 0 ? a.group : kFewMax;

  for (;;) {
    if (threadIdx.x == 0) s_item = atomicAdd(a.counter, 1);
    __syncthreads();
    const int item = s_item;
    if (item >= total) break;
    const int2 g = a.items[item];
    const int pb = a.pair_offsets[g.x] + g.y * group;
    const int pe0 = a.pair_offsets[g.x + 1];
    const int nq = (pe0 - pb) < kFewMax ? (pe0 - pb) : kFewMax;
    const long long rb = a.list_offsets[g.x];
    const long long re_all = a.list_offsets[g.x + 1];
    const long long re = (a.max_rows > 0 && re_all - rb > a.max_rows) ? rb + a.max_rows : re_all;
    // the item's queries (shared by the four warps)
    if (threadIdx.x < nq) {
      const int pr = a.pairs[pb + threadIdx.x];
      const int q = pr / a.P;
      s_slot[threadIdx.x] = pr;
      if (FLT) {
        s_qn[threadIdx.x] = a.pair_qn[pr];
        s_sc[threadIdx.x] = a.pair_sc[pr];
        s_bnd[threadIdx.x] = bound_key(a.pair_thr[pr]);
      } else {
        s_qn[threadIdx.x] = METRIC == MF_METRIC_L2 ? a.qnorms[q] : 0.0f;
        s_bnd[threadIdx.x] = a.bound ? bound_key(a.bound[q]) : kEmptyKey;
      }
    }
    for (int i = threadIdx.x; i < nq * d4; i += W * 32) {
      const int j = i / d4;
      const int pr = a.pairs[pb + j];
      float4 v = reinterpret_cast<const float4*>(a.xq + (long long)(pr / a.P) * d)[i - j * d4];
      if (FLT) {
        // s_q (q - c), exact scaling by a power of two
        const float4 c = reinterpret_cast<const float4*>(a.centroids + (long long)g.x * d)[i - j * d4];
        const float sq = a.pair_sq[pr];
        v = make_float4((v.x - c.x) * sq, (v.y - c.y) * sq, (v.z - c.z) * sq, (v.w - c.w) * sq);
      }
      qs[i] = v;
    }
    for (int i = lane; i < nq * kFewK; i += 32) lists[i] = kEmptyKey;
    __syncthreads();
    // lane j < nq: this warp's threshold and buffered count of query j
    unsigned long long bnd = lane < nq ? s_bnd[lane] : kEmptyKey;
    unsigned long long thr = bnd;
    int nbuf = 0;

    const float4* qv = qs + lane;  // this lane's column slice of each query
    const bool col_ok = lane < d4;
    // offers query j one key per lane (kEmptyKey: none): the keys below the
    // query's threshold go to its candidate buffer, which is merged into the
    // query's list first when they would overflow it
    auto insert = [&](int j, unsigned long long key) {
      const unsigned long long tj = __shfl_sync(0xffffffffu, thr, j);
      unsigned int m = __ballot_sync(0xffffffffu, key < tj);
      if (m == 0u) return;
      int nb = __shfl_sync(0xffffffffu, nbuf, j);
      unsigned long long* buf = bufs + j * 32;
      unsigned long long* list = lists + j * kFewK;
      if (nb + __popc(m) > 32) {
        const unsigned long long nk = merge_into_list<kFewK>(list, buf, nb, k, lane);
        const unsigned long long bj = __shfl_sync(0xffffffffu, bnd, j);
        const unsigned long long t2 = nk < bj ? nk : bj;
        if (lane == j) thr = t2;
        nb = 0;
        m = __ballot_sync(0xffffffffu, key < t2);
        if (m == 0u) {
          if (lane == j) nbuf = 0;
          return;
        }
      }
      if ((m >> lane) & 1u) buf[nb + __popc(m & lanemask_lt())] = key;
      if (lane == j) nbuf = nb + __popc(m);
      __syncwarp();
    };
    // rows r0 .. r0+15 (row i's column slice `lane` in xv[i]) against every query
    auto process = [&](const float4 (&xv)[kFewRows], long long r0) {
      const long long my_row = r0 + (lane >> 1);  // the row whose sum this lane ends with
      const bool rv = my_row < re && (lane & 1) == 0;
      const float xn = (METRIC == MF_METRIC_L2 && my_row < re) ? a.xnorms[my_row] : 0.0f;
#pragma unroll 1
      for (int j = 0; j < nq; ++j) {
        const float4 q4 = col_ok ? qv[j * d4] : make_float4(0.f, 0.f, 0.f, 0.f);
        float p[kFewRows];
#pragma unroll
        for (int i = 0; i < kFewRows; ++i) {
          float t = xv[i].x * q4.x;
          t = fmaf(xv[i].y, q4.y, t);
          t = fmaf(xv[i].z, q4.z, t);
          p[i] = fmaf(xv[i].w, q4.w, t);
        }
        const float dot = warp_transpose_reduce16(p, lane);
        const float dist = METRIC == MF_METRIC_L2 ? l2_from_dot(s_qn[j], xn, dot) : -dot;
        insert(j, rv ? make_key(dist, (unsigned int)my_row) : kEmptyKey);
      }
    };
    if constexpr (FLT) {
      // fp16 tensor-core products (mma.sync m16n8k16, fp32 accumulation). The
      // item's queries, rounded to fp16 as the tensor-core filter rounds them,
      // are the A operand (16 queries x 16 elements per K-step), 8 rows the B
      // operand. In K-steps 2p and 2p + 1, lane (g, t) = (lane / 4, lane % 4)
      // holds elements 32 p + 8 t .. + 3 and 32 p + 8 t + 4 .. + 7 of queries
      // g, g + 8 and of row g: both operands' K order is permuted alike, so the
      // products are the rows' dot products, and a row's B fragments for two
      // K-steps are one 16-byte load. The next 16 rows (and their norms) are
      // loaded before this step's products.
      const unsigned int full = 0xffffffffu;
      const int gq = lane >> 2, tq = lane & 3;
      const int nkp = (d + 31) >> 5;  // pairs of K-steps
      uint32_t af[kFewMaxD / 16][4];
#pragma unroll
      for (int s = 0; s < kFewMaxD / 16; ++s) {
        const int e0 = 32 * (s >> 1) + 8 * tq + 4 * (s & 1);
        float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
        if (e0 < d) {
          if (gq < nq) lo = qs[gq * d4 + (e0 >> 2)];
          if (gq + 8 < nq) hi = qs[(gq + 8) * d4 + (e0 >> 2)];
        }
        af[s][0] = few_pack_f16x2(lo.x, lo.y);
        af[s][1] = few_pack_f16x2(hi.x, hi.y);
        af[s][2] = few_pack_f16x2(lo.z, lo.w);
        af[s][3] = few_pack_f16x2(hi.z, hi.w);
      }
      const bool vlo = gq < nq, vhi = gq + 8 < nq;
      const float qn_lo = vlo ? s_qn[gq] : 0.f, sc_lo = vlo ? s_sc[gq] : 0.f;
      const float qn_hi = vhi ? s_qn[gq + 8] : 0.f, sc_hi = vhi ? s_sc[gq + 8] : 0.f;
      const uint4* hrows = reinterpret_cast<const uint4*>(a.xb);
      // rows r0 + 8 nt + gq (B fragments) and the norms of rows r0 + 8 nt + 2 tq + e
      auto load_step = [&](uint4 (&bv)[2][kFewMaxD / 32], float (&xn)[4], long long r0) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const long long r = r0 + 8 * nt + gq;
          const uint4* rp = hrows + ((r * d) >> 3) + tq;
#pragma unroll
          for (int p = 0; p < kFewMaxD / 32; ++p)
            bv[nt][p] = (r < re && 32 * p + 8 * tq < d) ? rp[4 * p] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const long long rx = r0 + 8 * nt + 2 * tq + e;
            xn[2 * nt + e] = rx < re ? a.xnorms[rx] : 0.0f;
          }
        }
      };
      // the row this lane gathers in the slow path (lanes 0..15: row r0 + lane)
      const int src_t = (lane & 7) >> 1, nt_l = (lane >> 3) & 1, e_l = lane & 1;
      const long long rstep = (long long)W * kFewRows;
      uint4 bv[2][kFewMaxD / 32];
      float xn[4];
      load_step(bv, xn, rb + (long long)warp * kFewRows);
      for (long long r0 = rb + (long long)warp * kFewRows; r0 < re; r0 += rstep) {
        uint4 bn[2][kFewMaxD / 32];
        float xnn[4];
        load_step(bn, xnn, r0 + rstep);
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int p = 0; p < kFewMaxD / 32; ++p) {
          if (p < nkp) {
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
              few_mma_f16(acc[nt], af[2 * p], bv[nt][p].x, bv[nt][p].y);
              few_mma_f16(acc[nt], af[2 * p + 1], bv[nt][p].z, bv[nt][p].w);
            }
          }
        }
        // acc[nt][2 h + e] (query gq + 8 h, row r0 + 8 nt + 2 tq + e) becomes
        // its upper bound u; does any of the lane's u pass its query's threshold?
        const unsigned long long t0 = __shfl_sync(full, thr, gq);
        const unsigned long long t1 = __shfl_sync(full, thr, gq + 8);
        const unsigned long long tlo = vlo ? t0 : 0ull, thi = vhi ? t1 : 0ull;
        bool plo = false, phi = false;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const long long r = r0 + 8 * nt + 2 * tq + e;
            acc[nt][e] = l2_from_dot(qn_lo, xn[2 * nt + e], acc[nt][e] * sc_lo);
            acc[nt][2 + e] = l2_from_dot(qn_hi, xn[2 * nt + e], acc[nt][2 + e] * sc_hi);
            if (r < re) {
              plo |= make_key(acc[nt][e], (unsigned int)r) < tlo;
              phi |= make_key(acc[nt][2 + e], (unsigned int)r) < thi;
            }
          }
        }
        const unsigned int mlo = __ballot_sync(full, plo);
        const unsigned int mhi = __ballot_sync(full, phi);
        if ((mlo | mhi) != 0u) {
          // the queries with a candidate: gather query j's 16 bounds to lanes
          // 0..15 (lane i: row r0 + i) and offer them
          unsigned int qm = 0u;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            if ((mlo >> (4 * g)) & 0xfu) qm |= 1u << g;
            if ((mhi >> (4 * g)) & 0xfu) qm |= 1u << (g + 8);
          }
          const long long rl = r0 + (lane & 15);
          while (qm != 0u) {
            const int j = __ffs(qm) - 1;
            qm &= qm - 1u;
            const int src = (j & 7) * 4 + src_t;
            const bool h = j >= 8;
            const float v00 = __shfl_sync(full, h ? acc[0][2] : acc[0][0], src);
            const float v01 = __shfl_sync(full, h ? acc[0][3] : acc[0][1], src);
            const float v10 = __shfl_sync(full, h ? acc[1][2] : acc[1][0], src);
            const float v11 = __shfl_sync(full, h ? acc[1][3] : acc[1][1], src);
            const float u = nt_l ? (e_l ? v11 : v10) : (e_l ? v01 : v00);
            insert(j, (lane < 16 && rl < re) ? make_key(u, (unsigned int)rl) : kEmptyKey);
          }
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int p = 0; p < kFewMaxD / 32; ++p) bv[nt][p] = bn[nt][p];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) xn[i] = xnn[i];
      }
    } else {
      for (long long r0 = rb + (long long)warp * kFewRows; r0 < re;
           r0 += (long long)W * kFewRows) {
        // rows r0 .. r0+15: load i brings row r0+i across the warp (coalesced)
        float4 xv[kFewRows];
#pragma unroll
        for (int i = 0; i < kFewRows; ++i) {
          const long long r = r0 + i;
          xv[i] = (r < re && col_ok) ? reinterpret_cast<const float4*>(a.xb + r * d)[lane]
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        process(xv, r0);
      }
    }
    // each warp folds its buffers into its lists; then warp (j mod 4) merges
    // the four warps' lists of query j and writes its k keys
    for (int j = 0; j < nq; ++j) {
      const int nb = __shfl_sync(0xffffffffu, nbuf, j);
      if (nb > 0) merge_into_list<kFewK>(lists + j * kFewK, bufs + j * 32, nb, k, lane);
    }
    __syncthreads();
    for (int j = warp; j < nq; j += W) {
      unsigned long long* list = lists + j * kFewK;
      for (int v = 0; v < W; ++v) {
        if (v == warp) continue;
        const unsigned long long* other = lists_all + v * kFewMax * (kFewK + 32) + j * kFewK;
        merge_into_list<kFewK>(list, other, k, k, lane);
      }
      const long long sj = s_slot[j];
      if (a.pair_cnt) {
        // compact: the kept keys (a sorted prefix), row positions, and their count
        const unsigned long long key = lane < k ? list[lane] : kEmptyKey;
        const unsigned int m = __ballot_sync(0xffffffffu, key != kEmptyKey);
        if (lane == 0) a.pair_cnt[sj] = __popc(m);
        if (key != kEmptyKey) {
          a.out_d[sj * a.out_stride + lane] = key_dist(key);
          a.out_l[sj * a.out_stride + lane] = (long long)key_index(key);
        }
      } else if (lane < k) {
        const unsigned long long key = list[lane];
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
        a.out_d[sj * k + lane] = dv;
        a.out_l[sj * k + lane] = lv;
      }
      __syncwarp();
    }
    __syncthreads();
  }
}

// Accumulation probe (a diagnostic, not on the search path): out (16 x 8) =
// A (16 x d) . B (8 x d)^T with mma.sync m16n8k16 (fp16 operands, fp32
// accumulation carried across the d / 16 K-steps in the C registers), the
// instruction the few-query filter pass uses. One warp; A and B row-major
// fp16, two elements per 32-bit word. Fragments: lane (g, t) = (lane / 4,
// lane % 4) holds A rows g and g + 8 at columns 2t, 2t + 1 and 2t + 8,
// 2t + 9, B row g at the same columns, and C rows g, g + 8 at columns 2t,
// 2t + 1.
__global__ void mma_f16_probe_kernel(const uint32_t* __restrict__ a,
                                     const uint32_t* __restrict__ b, int d,
                                     float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int w = d / 2;
  float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int k0 = 0; k0 < d; k0 += 16) {
    const int kw = k0 / 2 + t;
    const uint32_t af[4] = {a[g * w + kw], a[(g + 8) * w + kw], a[g * w + kw + 4],
                            a[(g + 8) * w + kw + 4]};
    few_mma_f16(c, af, b[g * w + kw], b[g * w + kw + 4]);
  }
  out[g * 8 + 2 * t] = c[0];
  out[g * 8 + 2 * t + 1] = c[1];
  out[(g + 8) * 8 + 2 * t] = c[2];
  out[(g + 8) * 8 + 2 * t + 1] = c[3];
}

}  // namespace

bool few_eligible(int metric, int d, int k) {
  return (metric == MF_METRIC_L2 || metric == MF_METRIC_INNER_PRODUCT) && d <= kFewMaxD &&
         d % 4 == 0 && k >= 1 && k <= kFewK;
}

int few_max_queries() { return kFewMax; }

int launch_few_scan(const ScanArgs& a, int metric, int64_t max_items, int device,
                    cudaStream_t stream) {
  MF_CHECK(few_eligible(metric, a.d, a.k), MF_ERR_INVALID_ARGS,
           "few-query scan does not take metric %d, d=%d, k=%d", metric, a.d, a.k);
  MF_CHECK(a.counter != nullptr && a.item_total != nullptr, MF_ERR_INVALID_ARGS,
           "few-query scan needs its items and a work counter");
  if (max_items <= 0) return MF_OK;
  const bool flt = a.pair_sq != nullptr;
  MF_CHECK(!flt || (metric == MF_METRIC_L2 && a.d <= kFewMaxD && a.d % 8 == 0 && a.pair_qn &&
                    a.pair_thr && a.pair_sc && a.pair_cnt && a.centroids),
           MF_ERR_INVALID_ARGS, "few-query filter scan: L2, d <= %d, per-pair arrays", kFewMaxD);
  // items capped at a few rows (the bound pass): kFewBoundWarps per item
  const bool bound_items = !flt && a.max_rows > 0 && a.max_rows <= kFewBoundRows;
  const int warps = bound_items ? kFewBoundWarps : kFewWarps;
  const size_t smem = FewSmem::block(a.d, warps);
  void (*fn)(const ScanArgs);
  if (flt)
    fn = few_scan_kernel<MF_METRIC_L2, true, kFewWarps>;
  else if (bound_items)
    fn = metric == MF_METRIC_L2 ? few_scan_kernel<MF_METRIC_L2, false, kFewBoundWarps>
                                : few_scan_kernel<MF_METRIC_INNER_PRODUCT, false, kFewBoundWarps>;
  else
    fn = metric == MF_METRIC_L2 ? few_scan_kernel<MF_METRIC_L2, false, kFewWarps>
                                : few_scan_kernel<MF_METRIC_INNER_PRODUCT, false, kFewWarps>;
  MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int per_sm = 0;
  MF_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, warps * 32, smem));
  if (per_sm < 1) per_sm = 1;
  long long grid = (long long)num_sms(device) * per_sm;
  if (grid > max_items) grid = max_items;
  MF_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(int), stream));
  ScopedTiming tm(a.max_rows > 0 ? "scan_topk_ivf_bound_small" : "scan_topk_ivf_small", stream);
  fn<<<(unsigned int)grid, warps * 32, smem, stream>>>(a);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_f16_probe_mma(const void* a, const void* b, int d, float* out,
                         cudaStream_t stream) {
  MF_CHECK(d >= 16 && d <= 1024 && d % 16 == 0, MF_ERR_INVALID_ARGS,
           "mma.sync probe: d=%d (a multiple of 16 in [16, 1024])", d);
  mma_f16_probe_kernel<<<1, 32, 0, stream>>>(reinterpret_cast<const uint32_t*>(a),
                                             reinterpret_cast<const uint32_t*>(b), d, out);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

}  // namespace mf
