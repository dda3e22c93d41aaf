// Tensor-core slab scan (sm_100a): L2 / inner-product top-k of a work item
// (<= 128 queries x a slab of rows) with the distance tile computed by tcgen05
// MMAs in 3xTF32 form, accumulators in TMEM, and a per-query top-k in the
// epilogue. Work items and outputs follow scan_kernel (mf_scan.cu), with
// query groups of 128.
//
// Operands (K-major, 128-byte swizzle, loaded by TMA without multicast):
//   A = the item's 128 queries (M = 128), B = a tile of BN database rows (N).
// The tensor core reads fp32 operands as tf32 by dropping the 13 low mantissa
// bits (truncation, checked on B200), so the raw fp32 arrays serve as the hi
// parts; the lo parts (x - trunc_tf32(x)) are precomputed: once per add for
// the database, once per search for the queries. Per K-step of 8:
//   D += A.B  +  A.B_lo  +  A_lo.B      (the dropped A_lo.B_lo term is ~2^-22)
//
// Warp roles (192 threads, one persistent CTA per SM, items taken dynamically):
//   warps 0-3  epilogue: thread t owns query row t of the tile (TMEM lane t),
//              reads its BN dot products, forms distances and keeps a sorted
//              per-thread top-k list in shared memory;
//   warp 4     TMA producer (one lane);
//   warp 5     TMEM allocation and MMA issue (one lane).
// Stages flow full -> MMA -> empty; accumulators flow accf -> epilogue -> acce
// through 512 / BN TMEM buffers, so the MMAs run up to that many tiles ahead of
// the epilogue. Every wait is bounded (mf_sm100.cuh).
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstring>
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

#ifdef MF_TC_PROFILE
// Per-role cycle counters (instrumented builds only).
__device__ unsigned long long g_tc_prof[20];
#define TQP(i, expr)                                       \
  do {                                                     \
    const long long _t0 = clock64();                       \
    expr;                                                  \
    atomicAdd(&g_tc_prof[i], (unsigned long long)(clock64() - _t0)); \
  } while (0)
// Epilogue thread 0 accumulates into locals (TQL) and adds them once at exit.
#define TQL(var, expr)                 \
  do {                                 \
    const long long _t0 = clock64();   \
    expr;                              \
    var += clock64() - _t0;            \
  } while (0)
#else
#define TQP(i, expr) expr
#define TQL(var, expr) expr
#endif

#if defined(MF_TC_PROFILE) || defined(MF_TC_TRACE)
#define MF_TC_STAMPS 1
// Per-tile and per-item clock stamps of the filter scan in the first kTrCtas
// CTAs (instrumented builds only): tiles [MMA accumulator free, MMA stage
// ready, MMA committed, epilogue got it, epilogue released it, its first
// accumulator chunk arrived, its first two chunks done, all chunks done,
// producer got the free stage (its loads issued), -], items
// [loader wrote A, MMA saw A, epilogue started, epilogue finished].
constexpr int kTrCtas = 2, kTrTiles = 4096, kTrItems = 1024;
__device__ long long g_tc_trace[kTrCtas][kTrTiles][10];
__device__ long long g_tc_trace_item[kTrCtas][kTrItems][4];
#define TQT(on, arr, idx, f, n)                                               \
  do {                                                                        \
    if ((on) && blockIdx.x < kTrCtas && (idx) < (n)) arr[blockIdx.x][idx][f] = clock64(); \
  } while (0)
#else
#define TQT(on, arr, idx, f, n) \
  do {                          \
  } while (0)
#endif

using namespace sm100;

// Warps: 0-3 epilogue, 4 producer, 5 MMA, (ATM) 6-9 query tile loader,
// (EW = 2) the second epilogue warpgroup, (filter scan) the second MMA issuer.
constexpr int kTqThreads = 192;
constexpr int kTqM = 128;          // queries per item = TMEM lanes
constexpr int kTqEpiThreads = 128;
constexpr int kTqMaxD = 1024;
constexpr int kTqK = 32;  // list slots per query row (k <= 32)
constexpr int kTqKBig = 128;  // list slots per query row for 32 < k <= 128
constexpr int kTqMaxSmem = 227 * 1024 - 512;
// All 512 TMEM columns hold accumulators: 512 / BN tiles in flight between
// the MMA warp and the epilogue (4 at BN = 128).
constexpr int kTqTmemCols = 512;
// Work items are taken from a global counter by the producer (largest items
// first, as the item arrays are ordered) and handed to the MMA warp and the
// epilogue warps through a ring of kTqQueue shared-memory slots. The ring is
// deeper than the tiles the producer can run ahead (stages + accumulators),
// so a run of one-tile items never stalls it.
constexpr int kTqQueue = 16;
constexpr int kTqMaxAcc = 4;
// With the query tile resident in tensor memory (d <= 128), warps 6-9 load
// it: 320 threads. Otherwise the query tile streams with the rows: 192.
constexpr int kTqThreadsAtm = 320;
constexpr int kTqMaxDAtm = 128;

struct TqLayout {
  int SA, KB, BN;  // KB: K-blocks of 128 bytes (32 fp32 or, with bf, 64 fp16)
  int ew;    // epilogue warpgroups (2: each takes half of every tile's columns)
  int atm;   // query tile in tensor memory (columns [0, 2*KB*32): hi then lo)
  int bf;    // 16-bit operands (filter scan): A in columns [0, KB*32), no residuals
  int nacc;  // accumulator buffers in tensor memory
  int acc0;  // first accumulator column
  size_t stage, a_hi, a_lo, b_hi, b_lo;  // offsets within a stage
  size_t lists, scratch, xn, rowthr, bars, total;
};

TqLayout tq_layout(int d, int kcap, int BN, int SA, bool atm, bool bf = false, int ew = 1) {
  TqLayout s;
  s.SA = SA;
  s.ew = ew;
  s.KB = bf ? (d + 63) / 64 : (d + 31) / 32;
  s.BN = BN;
  s.atm = atm ? 1 : 0;
  s.bf = bf ? 1 : 0;
  if (atm) {
    s.a_hi = s.a_lo = 0;  // unused: the query tile lives in tensor memory
    s.b_hi = 0;
    // bf: A in columns [0, KB*32), its norm-extension K-step in the next 32;
    // accumulators from the next multiple of 64
    s.acc0 = bf ? ((s.KB + 1) * 32 + 63) / 64 * 64 : 2 * s.KB * 32;
  } else {
    s.a_hi = 0;
    s.a_lo = kTqM * 128;
    s.b_hi = 2 * kTqM * 128;
    s.acc0 = 0;
  }
  s.nacc = (kTqTmemCols - s.acc0) / BN;
  if (s.nacc > kTqMaxAcc) s.nacc = kTqMaxAcc;
  s.b_lo = s.b_hi + size_t(BN) * 128;
  // the filter scan's stage holds a whole tile (all K-blocks, then the rows'
  // 32-byte norm extensions): one hand-off per tile
  s.stage = bf ? size_t(s.KB) * BN * 128 + size_t(BN) * 32 : s.b_lo + size_t(BN) * 128;
  size_t o = size_t(SA) * s.stage;
  s.lists = o;  // per epilogue warpgroup: 128 rows x kcap keys
  o += size_t(ew) * kTqM * kcap * 8;
  s.scratch = o;  // candidate buffers: 128 rows x 33 keys per warpgroup
  o += size_t(ew) * kTqM * 33 * 8;
  s.xn = o;  // row norms of the tile: a double buffer per epilogue warp
  o += size_t(ew) * (kTqEpiThreads / 32) * 2 * BN * 4;
  s.rowthr = o;  // ew > 1: each row's best k-th key over the warpgroups
  o += ew > 1 ? size_t(kTqM) * 8 : 0;
  s.bars = o;
  // mbarriers, then the item queue (kTqQueue slots of at most 48 bytes) and
  // the tensor-memory address, abort flag and sequence counters
  o += size_t(3 * SA + 2 * kTqMaxAcc + 2 * kTqQueue + 5) * 8 + kTqQueue * 48 + 32;
  s.total = o + 1024;
  return s;
}

struct TqMaps {
  CUtensorMap a_hi, a_lo, b_hi, b_lo;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Item geometry, computed by the producer and published with the item.
struct ItemDesc {
  long long rb, re;  // row slab
  int a_row0;        // first A row (queries) in the A tensor map
  int nq_item;       // valid queries (A rows) of this item
  int part;          // flat: the partial slot of this item's query tile
  int list;          // IVF: the item's list (-1 for flat)
};

// A queue slot: the item index (-1 ends the roles' loops) and its geometry.
struct QSlot {
  ItemDesc it;
  int item;
};

__device__ __forceinline__ ItemDesc item_desc(const ScanArgs& a, int item) {
  ItemDesc it;
  if (a.flat) {
    const int qt = item % a.nqt;
    const int s = item / a.nqt;
    it.a_row0 = qt * kTqM;
    const long long rem = a.nq - (long long)it.a_row0;
    it.nq_item = (int)(rem < kTqM ? rem : kTqM);
    it.rb = (long long)s * a.rows_per_split;
    const long long re = it.rb + a.rows_per_split;
    it.re = re < a.nb ? re : a.nb;
    it.part = s;
    it.list = -1;
  } else {
    it.part = 0;
    // a list's q queries are cut into ceil(q / 128) groups of nearly equal
    // size (group g: [p0 + g q / ng, p0 + (g + 1) q / ng))
    const int2 g = a.items[item];
    const int p0 = a.pair_offsets[g.x];
    const int q = a.pair_offsets[g.x + 1] - p0;
    const int ng = (q + kTqM - 1) / kTqM;
    const int pb = p0 + (int)(((long long)g.y * q) / ng);
    const int pe = p0 + (int)(((long long)(g.y + 1) * q) / ng);
    it.a_row0 = pb;
    it.nq_item = pe - pb;
    it.list = g.x;
    it.rb = a.list_offsets[g.x];
    const long long re = a.list_offsets[g.x + 1];
    it.re = (a.max_rows > 0 && re - it.rb > a.max_rows) ? it.rb + a.max_rows : re;
  }
  return it;
}

// Two fp32 rounded to fp16 (to nearest, ties to even), packed as one 32-bit
// tensor-memory column: the first in the low half.
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The filter scan's pipeline-critical waits (epilogue on an accumulator, MMA
// on a free accumulator or a landed stage) spin without a suspend hint.
#ifndef MF_TC_SPIN
#define MF_TC_SPIN 0
#endif
constexpr bool kTcSpin = MF_TC_SPIN != 0;
constexpr bool kTcSpinProducer = MF_TC_SPIN > 1;  // the producer's waits on free stages too

// Survivors per lane up to which a chunk's keys are built by each lane's own
// loop over its set bits; past it, by one pass over all 32 columns.
constexpr unsigned int kTqSerialSurvivors = 6;

// r[j] for a run-time j without indexing the register array (which would put
// it in local memory): five levels of selects on the bits of j.
__device__ __forceinline__ uint32_t select32(const uint32_t (&r)[32], int j) {
  uint32_t a[16], b[8], c[4], d[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (j & 1) ? r[2 * i + 1] : r[2 * i];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = (j & 2) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = (j & 4) ? b[2 * i + 1] : b[2 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) d[i] = (j & 8) ? c[2 * i + 1] : c[2 * i];
  return (j & 16) ? d[1] : d[0];
}

// Packed pairs of fp32 (Blackwell's two-wide fp32 add / sub / fma): each half
// is rounded like the scalar instruction.
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
  return static_cast<unsigned long long>(__float_as_uint(lo)) |
         (static_cast<unsigned long long>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b,
                                                   unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Accept mask of a 32-column chunk: bit j is set iff column j's distance is
// <= thr_d (the row's current k-th distance, its bound, or +inf while open)
// and j < nvalid. For L2, t = (qn + xn) - 2 dot is formed as l2_from_dot forms
// it before its clamp at 0 (doubling is exact, so the FMA rounds once, like the
// subtraction; m2 is -2, or -2 times the power-of-two scale of the filter
// scan's accumulators, so m2 * acc is still exactly -2 dot); thr_d >= 0, so
// t <= thr_d iff the clamped distance is. The
// sign bit of thr_d - t (+0 when equal) is shifted into a reject mask. Columns
// go two at a time through the packed fp32 pipe, in four independent shift
// chains of 8 columns joined at the end.
template <int METRIC>
__device__ __forceinline__ unsigned int tq_accept(const uint32_t (&r)[32], const float* xs,
                                                  float qn, float m2s, float thr_d, int nvalid) {
  unsigned int rej[4] = {0u, 0u, 0u, 0u};
  const unsigned long long thr2 = pack2(thr_d, thr_d);
  float x[32];
  if (METRIC == MF_METRIC_L2) {
    // xs is 16-byte aligned (chunk offsets are multiples of 32 floats)
    const float4* x4 = reinterpret_cast<const float4*>(xs);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = x4[i];
      x[4 * i] = t.x;
      x[4 * i + 1] = t.y;
      x[4 * i + 2] = t.z;
      x[4 * i + 3] = t.w;
    }
  }
  const unsigned long long qn2 = pack2(qn, qn);
  const unsigned long long m2 = pack2(m2s, m2s);
#pragma unroll
  for (int p = 3; p >= 0; --p) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int j = 8 * g + 2 * p;  // columns j (low half) and j + 1 (high half)
      const unsigned long long dot2 =
          static_cast<unsigned long long>(r[j]) | (static_cast<unsigned long long>(r[j + 1]) << 32);
      unsigned long long diff2;
      if (METRIC == MF_METRIC_L2)
        diff2 = sub2(thr2, fma2(m2, dot2, add2(qn2, pack2(x[j], x[j + 1]))));
      else
        diff2 = add2(thr2, dot2);
      rej[g] = __funnelshift_l(static_cast<unsigned int>(diff2 >> 32), rej[g], 1);
      rej[g] = __funnelshift_l(static_cast<unsigned int>(diff2), rej[g], 1);
    }
  }
  const unsigned int all = rej[0] | (rej[1] << 8) | (rej[2] << 16) | (rej[3] << 24);
  const unsigned int in_range = nvalid >= 32 ? 0xffffffffu : ((1u << nvalid) - 1u);
  return ~all & in_range;
}

// The largest of 32 fp32 values as a tree of three-input maxima (no NaN
// among them: the accumulators of finite operands).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max32(const uint32_t (&r)[32]) {
  float l1[11];
#pragma unroll
  for (int i = 0; i < 10; ++i)
    l1[i] = max3f(__uint_as_float(r[3 * i]), __uint_as_float(r[3 * i + 1]),
                  __uint_as_float(r[3 * i + 2]));
  l1[10] = fmaxf(__uint_as_float(r[30]), __uint_as_float(r[31]));
  const float a = max3f(l1[0], l1[1], l1[2]);
  const float b = max3f(l1[3], l1[4], l1[5]);
  const float c = max3f(l1[6], l1[7], l1[8]);
  return max3f(max3f(a, b, c), l1[9], l1[10]);
}

// Accept mask of a 32-column chunk of the filter scan, whose accumulators
// already hold s_q s_l (dot - rn_x / 2): bit j is set iff acc_j >= tau (the
// row's threshold moved to the accumulator's scale, lowered by a margin so
// that every column the exact form would keep passes) and j < nvalid. One
// packed subtraction per two columns; the sign bit of acc - tau (+0 when
// equal) goes into the reject mask, in four independent chains.
__device__ __forceinline__ unsigned int tq_accept_acc(const uint32_t (&r)[32], float tau,
                                                      int nvalid) {
  unsigned int rej[4] = {0u, 0u, 0u, 0u};
  const unsigned long long tau2 = pack2(tau, tau);
#pragma unroll
  for (int p = 3; p >= 0; --p) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int j = 8 * g + 2 * p;
      const unsigned long long acc2 =
          static_cast<unsigned long long>(r[j]) | (static_cast<unsigned long long>(r[j + 1]) << 32);
      const unsigned long long diff2 = sub2(acc2, tau2);
      rej[g] = __funnelshift_l(static_cast<unsigned int>(diff2 >> 32), rej[g], 1);
      rej[g] = __funnelshift_l(static_cast<unsigned int>(diff2), rej[g], 1);
    }
  }
  const unsigned int all = rej[0] | (rej[1] << 8) | (rej[2] << 16) | (rej[3] << 24);
  const unsigned int in_range = nvalid >= 32 ? 0xffffffffu : ((1u << nvalid) - 1u);
  return ~all & in_range;
}

// CONV (with ATM only): the rows' tf32 residuals are derived in shared memory
// from the loaded fp32 tile instead of being loaded (no residual array).
// FLT (with ATM, L2, IVF only): the filter scan. One fp16 MMA per K-step of 16
// replaces the three tf32 ones; A = fp16(s_q (query - list centroid)) in
// tensor memory, B = the rows' fp16 residuals against that centroid (scaled
// by the list's power of two s_l); per pair, the query norm, the bound, s_q
// and 1 / (s_q s_l) come from a.pair_qn / pair_thr / pair_sq / pair_sc, and
// each pair's kept slots are written with their count (a.pair_cnt).
//
// KC: list slots per query row: kTqK (k <= 32) or kTqKBig (k <= 128, with
// 64-row tiles so the larger lists fit in shared memory beside the stages).
//
// EW: epilogue warpgroups. With 2 (the filter scan), warps 10-13 form a second
// epilogue warpgroup: each group takes half of every tile's columns with its
// own per-row lists and candidate buffers, the rows' thresholds are shared
// through shared memory (any group's k-th key bounds the union's), and at the
// end of an item the second group's lists are merged into the first's, which
// writes the results. Two warps per SM sub-partition then hide each other's
// latencies in the per-column filter that bounds this scan.
template <int METRIC, int BN, bool ATM, bool CONV, bool FLT = false, int KC = kTqK, int EW = 1>
__global__ void __launch_bounds__((ATM ? kTqThreadsAtm : kTqThreads) + (EW - 1) * kTqEpiThreads +
                                      (FLT ? 32 : 0), 1)
    tq_scan_kernel(const ScanArgs a, const __grid_constant__ TqMaps maps, const TqLayout L) {
  static_assert(EW == 1 || (EW == 2 && FLT && ATM && KC == kTqK),
                "two epilogue warpgroups are built for the filter scan only");
  extern __shared__ unsigned char smem_raw[];
  const int NACC = L.nacc;
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned long long* lists = reinterpret_cast<unsigned long long*>(base + L.lists);
  float* xn_s = reinterpret_cast<float*>(base + L.xn);
  unsigned long long* cbuf = reinterpret_cast<unsigned long long*>(base + L.scratch);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bars);
  uint64_t* empty = full + L.SA;
  uint64_t* conv = empty + L.SA;  // ATM: the stage's residual tile is written
  uint64_t* accf = conv + L.SA;
  uint64_t* acce = accf + kTqMaxAcc;
  uint64_t* qfull = acce + kTqMaxAcc;
  uint64_t* qempty = qfull + kTqQueue;
  uint64_t* afull = qempty + kTqQueue;  // query tile written to tensor memory
  uint64_t* afree = afull + 1;          // MMAs of the previous item done with it
  uint64_t* mdone = afree + 1;          // every MMA of this CTA has completed
  uint64_t* wgdone = mdone + 1;         // EW > 1: the second group's lists are final
  uint64_t* wgfree = wgdone + 1;        // EW > 1: the first group has read them
  unsigned long long* rowthr = reinterpret_cast<unsigned long long*>(base + L.rowthr);
  QSlot* s_q = reinterpret_cast<QSlot*>(wgfree + 1);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_q + kTqQueue);
  int* s_abort = reinterpret_cast<int*>(s_tmem + 1);
  uint32_t* s_seq = reinterpret_cast<uint32_t*>(s_abort + 1);  // [1]: stages issued

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  // The filter scan has two MMA issuers (alternate tiles; its one stage per
  // tile with an even ring keeps every stage's barriers with one issuer, so
  // each is waited on in phase order); the other variants have one.
  constexpr bool kTwoIss = FLT;
  constexpr int kMma2Warp = kTwoIss ? 10 + (EW - 1) * 4 : -1;
  const int SA = L.SA;
  const int KB = L.KB;
  const int k = a.k;
  const int total = a.flat ? a.nqt * a.P : *a.item_total;
  // ATM: the rows' fp32 tile and residual tile are loaded (CONV: only the fp32
  // tile; the loader warps derive its tf32 residual in shared memory).
  constexpr uint32_t kStageTx = FLT ? BN * 128
                                : ATM ? (CONV ? BN * 128 : 2 * BN * 128)
                                      : 2 * kTqM * 128 + 2 * BN * 128;

#ifdef MF_TC_PROFILE
  const long long _tk = clock64();
#endif
  if (warp == 5) {
    tmem_alloc(s_tmem, kTqTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < SA; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
      mbar_init(&conv[i], kTqM);
    }
    for (int i = 0; i < NACC; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], kTqEpiThreads * EW);
    }
    // readers of each queue slot: the MMA lane(s) and one lane per epilogue
    // (and loader) warp
    for (int i = 0; i < kTqQueue; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], (ATM ? 9 : 5) + 4 * (EW - 1) + (kTwoIss ? 1 : 0));
    }
    mbar_init(afull, kTqM);
    mbar_init(afree, kTwoIss ? 2 : 1);  // one commit from each MMA issuer
    mbar_init(mdone, kTwoIss ? 2 : 1);
    mbar_init(wgdone, 4);
    mbar_init(wgfree, 4);
    *s_abort = 0;
    s_seq[0] = 0;
    s_seq[1] = 0;
    fence_mbar_init();
  }
  if (EW > 1 && tid < kTqM) rowthr[tid] = kEmptyKey;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      if (!ATM) {
        prefetch_tensormap(&maps.a_hi);
        prefetch_tensormap(&maps.a_lo);
      }
      prefetch_tensormap(&maps.b_hi);
      if (!CONV) prefetch_tensormap(&maps.b_lo);  // FLT: the norm extensions
      uint32_t seq = 0;
      // flat, chunked: this CTA's run of (query tile x 128-row tile) tiles
      const bool chunked = a.flat && a.chunk_tiles > 0;
      long long cg = chunked ? (long long)blockIdx.x * a.chunk_tiles : 0;
      long long cend = 0;
      if (chunked) {
        const long long all = (long long)a.nqt * a.tiles_per_qt;
        cend = cg + a.chunk_tiles < all ? cg + a.chunk_tiles : all;
      }
      for (uint32_t qi = 0;; ++qi) {
        // take the next item and publish it (-1 ends every role's loop)
        const int qs = qi % kTqQueue;
        if (qi >= (uint32_t)kTqQueue)
          mbar_wait(&qempty[qs], ((qi / kTqQueue) - 1) & 1, s_abort, &g_device_error);
        int item = -1;
        ItemDesc it{};
        if (chunked) {
          // the next piece of the run: up to the end of its query tile
          if (!*s_abort && cg < cend) {
            const long long qt = cg / a.tiles_per_qt;
            const long long t0 = cg - qt * a.tiles_per_qt;
            long long t1 = t0 + (cend - cg);
            if (t1 > a.tiles_per_qt) t1 = a.tiles_per_qt;
            it.a_row0 = (int)(qt * kTqM);
            const long long rem = a.nq - (long long)it.a_row0;
            it.nq_item = (int)(rem < kTqM ? rem : kTqM);
            it.rb = t0 * kScanTR;
            const long long re = t1 * kScanTR;
            it.re = re < a.nb ? re : a.nb;
            it.part = (int)(blockIdx.x - (qt * a.tiles_per_qt) / a.chunk_tiles);
            it.list = -1;
            item = (int)qi;
            cg += t1 - t0;
          }
        } else {
          item = *s_abort ? -1 : atomicAdd(a.counter, 1);
          if (item >= total) item = -1;
          if (item >= 0) it = item_desc(a, item);
        }
        s_q[qs].it = it;
        s_q[qs].item = item;
        mbar_arrive(&qfull[qs]);
        if (item < 0) break;
        const long long nrows = it.re > it.rb ? it.re - it.rb : 0;
        const int nT = (int)((nrows + BN - 1) / BN);
        const int kps = FLT ? KB : 1;  // K-blocks per stage
        for (int t = 0; t < nT && !*s_abort; ++t) {
          for (int kb0 = 0; kb0 < KB; kb0 += kps) {
            const int s = seq % SA;
            bool ok = true;
            if (seq >= (uint32_t)SA)
              TQP(0, ok = mbar_wait<FLT && kTcSpinProducer>(&empty[s], ((seq / SA) - 1) & 1,
                                                            s_abort, &g_device_error));
            if (!ok) break;
            TQT(FLT, g_tc_trace, seq, 8, kTrTiles);
            unsigned char* st = base + size_t(s) * L.stage;
            mbar_arrive_expect_tx(&full[s], FLT ? (uint32_t)(KB * BN * 128 + BN * 32) : kStageTx);
            const int yb = (int)(it.rb + (long long)t * BN);
            for (int kb = kb0; kb < kb0 + kps; ++kb) {
              const int x = kb * (FLT ? 64 : 32);
              if (!ATM) {
                tma_load_2d(st + L.a_hi, &maps.a_hi, x, it.a_row0, &full[s]);
                tma_load_2d(st + L.a_lo, &maps.a_lo, x, it.a_row0, &full[s]);
              }
              tma_load_2d(st + L.b_hi + size_t(kb - kb0) * BN * 128, &maps.b_hi, x, yb, &full[s]);
              if (!CONV && !FLT) tma_load_2d(st + L.b_lo, &maps.b_lo, x, yb, &full[s]);
            }
            // FLT: the tile's norm extensions (32 bytes a row, x = 0)
            if (FLT) tma_load_2d(st + size_t(KB) * BN * 128, &maps.b_lo, 0, yb, &full[s]);
            ++seq;
          }
        }
      }
      s_seq[1] = seq;
    }
  } else if (warp == 5 || warp == kMma2Warp) {
    // ---------------------------------------------------------------- MMA
    // The filter scan's two issuing threads take alternate tiles. A wait on a
    // barrier, even one already complete, stalls the issuing thread for about
    // three MMAs' time while the tensor pipe queues about one, so with one
    // issuer the pipe sat idle through every tile's two waits; with two, one
    // issuer's waits overlap the other's MMAs.
    if (lane == 0) {
      const uint32_t me = warp == 5 ? 0u : 1u;
      constexpr uint32_t idesc = FLT ? idesc_f16(kTqM, BN) : idesc_tf32(kTqM, BN);
      uint32_t seq = 0, tt = 0;
      for (uint32_t qi = 0;; ++qi) {
        const int qs = qi % kTqQueue;
        bool qok = true;
        TQP(16, qok = mbar_wait(&qfull[qs], (qi / kTqQueue) & 1, s_abort, &g_device_error));
        if (!qok) break;
        const int item = s_q[qs].item;
        const ItemDesc it = s_q[qs].it;
        mbar_arrive(&qempty[qs]);
        if (item < 0) break;
        const long long nrows = it.re > it.rb ? it.re - it.rb : 0;
        const int nT = (int)((nrows + BN - 1) / BN);
        if (ATM) {
          // this item's query tile is in tensor memory
          bool aok = true;
          TQP(17, aok = mbar_wait(afull, qi & 1, s_abort, &g_device_error));
          if (!aok) break;
          TQT(FLT, g_tc_trace_item, qi, 1, kTrItems);
          tc_fence_after();
        }
        for (int t = 0; t < nT; ++t, ++tt) {
          if (kTwoIss && (tt & 1u) != me) {  // the other issuer's tile (one stage)
            ++seq;
            continue;
          }
          const int b = tt % NACC;
          if (tt >= (uint32_t)NACC)
            TQP(1, mbar_wait<FLT && kTcSpin>(&acce[b], ((tt / NACC) - 1) & 1, s_abort,
                                             &g_device_error));
          TQT(FLT, g_tc_trace, tt, 0, kTrTiles);
          tc_fence_after();
          const uint32_t dt = tmem + L.acc0 + b * BN;
          const int kps = FLT ? KB : 1;  // K-blocks per stage
          for (int kb0 = 0; kb0 < KB; kb0 += kps, ++seq) {
            const int s = seq % SA;
            TQP(2, mbar_wait<FLT && kTcSpin>(CONV ? &conv[s] : &full[s], (seq / SA) & 1, s_abort,
                                             &g_device_error));
            TQT(FLT, g_tc_trace, tt, 1, kTrTiles);
            tc_fence_after();
            const uint32_t st = smem_u32(base + size_t(s) * L.stage);
#ifdef MF_TC_PROFILE
            const long long _tm = clock64();
#endif
            for (int kb = kb0; kb < kb0 + kps; ++kb) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t off = kk * 32;  // 8 tf32 (or 16 fp16) of K per MMA
              const uint64_t bh =
                  desc_k_sw128(st + L.b_hi + (uint32_t)((kb - kb0) * BN * 128) + off);
              const uint64_t bl = desc_k_sw128(st + L.b_lo + off);
              if (FLT) {
                // 16 fp16 of K = 8 columns of the query tile
                mma_f16_ts(dt, tmem + kb * 32 + kk * 8, bh, idesc, !(kb == 0 && kk == 0));
              } else if (ATM) {
                // A columns: hi at [0, KB*32), lo at [KB*32, 2*KB*32)
                const uint32_t ah = tmem + kb * 32 + kk * 8;
                const uint32_t al = ah + KB * 32;
                mma_tf32_ts(dt, ah, bh, idesc, !(kb == 0 && kk == 0));
                mma_tf32_ts(dt, ah, bl, idesc, true);
                mma_tf32_ts(dt, al, bh, idesc, true);
              } else {
                const uint64_t ah = desc_k_sw128(st + L.a_hi + off);
                const uint64_t al = desc_k_sw128(st + L.a_lo + off);
                mma_tf32(dt, ah, bh, idesc, !(kb == 0 && kk == 0));
                mma_tf32(dt, ah, bl, idesc, true);
                mma_tf32(dt, al, bh, idesc, true);
              }
            }
            }
            if (FLT)  // the norm-extension K-step: acc += A_e (hi + lo) of each row
              mma_f16_ts(dt, tmem + KB * 32, desc_k_sw32(st + (uint32_t)(KB * BN * 128)), idesc,
                         true);
            mma_commit(&empty[s]);
#ifdef MF_TC_PROFILE
            atomicAdd(&g_tc_prof[8], (unsigned long long)(clock64() - _tm));
#endif
          }
          mma_commit(&accf[b]);
          TQT(FLT, g_tc_trace, tt, 2, kTrTiles);
        }
        // the query tile may be overwritten once this item's MMAs (both
        // issuers') complete
        if (ATM) mma_commit(afree);
      }
      // lets the teardown free tensor memory only after the last MMA, also when
      // a role gave up early
      mma_commit(mdone);
    }
  } else if (ATM && warp >= 6 && warp < 10) {
    // ------------------------------------------ query tile loader + residuals
    // Thread t of warps 6-9 owns TMEM lane 32*(warp%4)+lane = query row of
    // the item. Per item it writes the query tile to its lane once the
    // previous item's MMAs are done (hi = the raw fp32, which the tensor core
    // truncates to tf32, in columns [0, KB*32); lo = x - trunc(x) in
    // [KB*32, 2*KB*32); zero past d), then reads the next item's query rows
    // into registers (their latency overlaps what follows), then derives the
    // tf32 residual of every row stage of the item as it lands:
    // lo = x - trunc(x), elementwise at the same swizzled offset, so only the
    // rows' fp32 tile crosses HBM.
    const int row = 32 * (warp & 3) + lane;
    const int cid = (warp - 6) * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
    constexpr int kMaxV = FLT ? 1 : kTqMaxDAtm / 4;
    float4 v[kMaxV];
    // FLT: the row s_q (q - c) is packed to fp16 as it arrives (half the
    // registers of the fp32 row the tf32 form keeps)
    uint32_t hq[FLT ? kTqMaxDAtm / 2 : 1];
    // FLT: the row's norm-extension element A_e (two copies, as fp16)
    uint32_t ae2 = 0u;
    // FLT: s_q (the query row minus the item's list centroid)
    auto fetch = [&](const ItemDesc& it) {
      const float* src = nullptr;
      const float* cen = nullptr;
      float sq = 1.0f;
      ae2 = 0u;
      if (row < it.nq_item) {
        const int pr = a.flat ? 0 : a.pairs[it.a_row0 + row];
        const long long q = a.flat ? (long long)it.a_row0 + row : pr / a.P;
        src = a.xq + q * a.d;
        if (FLT) {
          cen = a.centroids + (long long)it.list * a.d;
          sq = a.pair_sq[pr];
          const float ae = a.pair_ae[pr];  // a power of two (or 0): exact in fp16
          ae2 = pack_f16x2(ae, ae);
        }
      }
      if constexpr (FLT) {
#pragma unroll
        for (int i = 0; i < kTqMaxDAtm / 4; ++i) {
          float4 e = make_float4(0.f, 0.f, 0.f, 0.f);
          if (src != nullptr && 4 * i < a.d) {
            const float4 x = *reinterpret_cast<const float4*>(src + 4 * i);
            const float4 c = *reinterpret_cast<const float4*>(cen + 4 * i);
            e = make_float4((x.x - c.x) * sq, (x.y - c.y) * sq, (x.z - c.z) * sq,
                            (x.w - c.w) * sq);
          }
          hq[2 * i] = pack_f16x2(e.x, e.y);
          hq[2 * i + 1] = pack_f16x2(e.z, e.w);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kMaxV; ++i) {
          v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (src != nullptr && 4 * i < a.d) v[i] = *reinterpret_cast<const float4*>(src + 4 * i);
        }
      }
    };
    auto take = [&](uint32_t qi, int& item, ItemDesc& it) -> bool {
      const int qs = qi % kTqQueue;
      if (!mbar_wait(&qfull[qs], (qi / kTqQueue) & 1, s_abort, &g_device_error)) return false;
      item = s_q[qs].item;
      it = s_q[qs].it;
      __syncwarp();
      if (lane == 0) mbar_arrive(&qempty[qs]);
      return true;
    };
    uint32_t cseq = 0;
    int item;
    ItemDesc it;
    if (take(0, item, it) && item >= 0) {
      fetch(it);
      for (uint32_t qi = 0;; ++qi) {
        if (qi > 0 && !mbar_wait(afree, (qi - 1) & 1, s_abort, &g_device_error)) break;
        tc_fence_after();
        if constexpr (FLT) {
          // 64 fp16 of K per 32 columns
#pragma unroll
          for (int c = 0; c < kTqMaxDAtm / 64; ++c) {
            if (c < KB) {
              uint32_t pk[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) pk[i] = hq[c * 32 + i];
              tmem_st32(lane_base + c * 32, pk);
            }
          }
          {
            // the norm-extension K-step: [A_e, A_e, 0, ...] (16 fp16)
            uint32_t pk[32];
            pk[0] = ae2;
#pragma unroll
            for (int i = 1; i < 32; ++i) pk[i] = 0u;
            tmem_st32(lane_base + KB * 32, pk);
          }
        }
        if constexpr (!FLT) {
#pragma unroll
        for (int c = 0; c < kTqMaxDAtm / 32; ++c) {
          if (c < KB) {
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float e[4] = {v[c * 8 + i].x, v[c * 8 + i].y, v[c * 8 + i].z, v[c * 8 + i].w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float h, l;
                split_tf32(e[j], h, l);
                hi[4 * i + j] = __float_as_uint(e[j]);
                lo[4 * i + j] = __float_as_uint(l);
                (void)h;
              }
            }
            tmem_st32(lane_base + c * 32, hi);
            tmem_st32(lane_base + KB * 32 + c * 32, lo);
          }
        }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(afull);
        if (cid == 0) TQT(FLT, g_tc_trace_item, qi, 0, kTrItems);
        // This item's row stages. The next item's queries are fetched as soon
        // as it is published (checked without blocking between stages: the
        // producer publishes it only after issuing this item's stages, which
        // need these conversions to free the ring), else after the loop.
        const ItemDesc cur = it;
        int nitem = -1;
        ItemDesc nit{};
        bool have_next = false, more = true;
        const uint32_t nq = qi + 1;
        const long long nrows = cur.re > cur.rb ? cur.re - cur.rb : 0;
        const int nst = CONV ? (int)((nrows + BN - 1) / BN) * KB : 0;
        bool ok = true;
        for (int j = 0; j < nst && ok; ++j, ++cseq) {
          // warp-uniform: lane 0's view decides, take() syncs the warp
          if (!have_next &&
              __shfl_sync(0xffffffffu, (int)mbar_test(&qfull[nq % kTqQueue], (nq / kTqQueue) & 1),
                          0)) {
            more = take(nq, nitem, nit);
            have_next = true;
            if (more && nitem >= 0) fetch(nit);
          }
          const int sidx = cseq % SA;
          if (!mbar_wait(&full[sidx], (cseq / SA) & 1, s_abort, &g_device_error)) {
            ok = false;
            break;
          }
          unsigned char* st = base + size_t(sidx) * L.stage;
          const float4* hi4 = reinterpret_cast<const float4*>(st + L.b_hi);
          float4* lo4 = reinterpret_cast<float4*>(st + L.b_lo);
#pragma unroll
          for (int i = 0; i < BN * 32 / 4 / kTqM; ++i) {
            const float4 x = hi4[cid + i * kTqM];
            float4 h, l;
            split_tf32(x.x, h.x, l.x);
            split_tf32(x.y, h.y, l.y);
            split_tf32(x.z, h.z, l.z);
            split_tf32(x.w, h.w, l.w);
            lo4[cid + i * kTqM] = l;
          }
          fence_proxy_async_smem();
          mbar_arrive(&conv[sidx]);
        }
        if (!ok) break;
        if (!have_next) {
          more = take(nq, nitem, nit);
          if (more && nitem >= 0) fetch(nit);
        }
        if (!more || nitem < 0) break;
        item = nitem;
        it = nit;
      }
    }
  } else {
    // ----------------------------------------------------------- epilogue
    // Lane l of epilogue warp w owns query row 32w+l: it reads that row of the
    // accumulator, filters the distances against the row's k-th best key
    // (thr, a register) and appends survivors to the row's 32-slot candidate
    // buffer. A full buffer is sorted and merged by the whole warp into the
    // row's top-k list (sorted, one key per lane, in shared memory).
    uint32_t tt = 0;
#ifdef MF_TC_PROFILE
    long long p_wait = 0, p_loop = 0, p_merge = 0, p_tiles = 0, p_nmerge = 0, p_out = 0;
    long long p_stage = 0, p_filter = 0, p_append = 0, p_tld = 0, p_nappend = 0;
    const long long p_start = clock64();
#endif
    // eg: this warp's epilogue group; eq: its quarter of the tensor-memory
    // lanes (a warp reads lanes 32 (warp % 4) ...); erow: this thread's row of
    // the tile. Group eg takes columns [cbeg, cend) of every tile.
    const int eg = EW > 1 && warp >= 10 ? 1 : 0;
    const int eq = warp & 3;
    const int erow = 32 * eq + lane;
    const int ewarp = eg * 4 + eq;
    constexpr int kCols = BN / EW;
    const int cbeg = eg * kCols;
    const int cend = cbeg + kCols;
    unsigned long long* my_lists = lists + (size_t)eg * kTqM * KC + (size_t)(eq * 32) * KC;
    unsigned long long* my_bufs = cbuf + (size_t)eg * kTqM * 33 + (size_t)(eq * 32) * 33;
    unsigned long long* own_buf = my_bufs + lane * 33;
    // Merges the buffered candidates of the rows in `who` (a warp-uniform
    // lane mask) into their sorted lists, two rows at a time so the shuffles
    // of the two sorting networks overlap. Each merged row's lane clears its
    // count and lowers its threshold to min(new k-th key, bound).
    // The merged rows' threads publish their new k-th distance when the
    // pieces of a flat query tile share them (a.share; qrow: the calling
    // thread's own query).
    auto merge_rows = [&](unsigned int who, int& cnt_reg, unsigned long long& thr_reg,
                          unsigned long long bnd, int qrow) {
      if constexpr (KC > kTqK) {
        // longer lists: one row at a time, the rank merge of the SIMT scan
        // (sorted batch; every element's new place is its old one plus its
        // rank in the other sequence)
        while (who) {
          const int s0 = __ffs(who) - 1;
          who &= who - 1;
          const int n0 = __shfl_sync(0xffffffffu, cnt_reg, s0);
          const unsigned long long nk =
              merge_into_list<KC>(my_lists + (size_t)s0 * KC, my_bufs + s0 * 33, n0, k, lane);
          if (lane == s0) {
            thr_reg = nk < bnd ? nk : bnd;
            cnt_reg = 0;
            if (a.share && nk != kEmptyKey) atomicMin(a.share + qrow, (unsigned int)(nk >> 32));
          }
          __syncwarp();
        }
        return;
      }
      while (who) {
        const int s0 = __ffs(who) - 1;
        who &= who - 1;
        int s1 = -1;
        if (who) {
          s1 = __ffs(who) - 1;
          who &= who - 1;
        }
        const int s1r = s1 < 0 ? s0 : s1;
        const int n0 = __shfl_sync(0xffffffffu, cnt_reg, s0);
        const int n1 = s1 < 0 ? 0 : __shfl_sync(0xffffffffu, cnt_reg, s1r);
        unsigned long long c[2], x[2];
        c[0] = lane < n0 ? my_bufs[s0 * 33 + lane] : kEmptyKey;
        c[1] = lane < n1 ? my_bufs[s1r * 33 + lane] : kEmptyKey;
        unsigned long long* l0 = my_lists + (size_t)s0 * KC;
        unsigned long long* l1 = my_lists + (size_t)s1r * KC;
        const unsigned long long e0 = l0[lane];  // ascending; kEmpty past k
        const unsigned long long e1 = l1[lane];
        warp_sort32_n<2>(c, lane);
        // the 32 smallest of a list and a sorted batch: elementwise min against
        // the batch reversed is bitonic; five half-cleaners sort it ascending
        x[0] = __shfl_sync(0xffffffffu, c[0], 31 - lane);
        x[1] = __shfl_sync(0xffffffffu, c[1], 31 - lane);
        x[0] = e0 < x[0] ? e0 : x[0];
        x[1] = e1 < x[1] ? e1 : x[1];
        warp_bitonic_clean32_n<2>(x, lane);
        if (lane >= k) x[0] = x[1] = kEmptyKey;
        l0[lane] = x[0];
        if (s1 >= 0) l1[lane] = x[1];
        const unsigned long long nk0 = __shfl_sync(0xffffffffu, x[0], k - 1);
        const unsigned long long nk1 = __shfl_sync(0xffffffffu, x[1], k - 1);
        if (lane == s0) {
          thr_reg = nk0 < bnd ? nk0 : bnd;
          cnt_reg = 0;
          if (!FLT && a.share && nk0 != kEmptyKey)
            atomicMin(a.share + qrow, (unsigned int)(nk0 >> 32));
          if (EW > 1 && nk0 != kEmptyKey) atomicMin(rowthr + erow, nk0);
        }
        if (lane == s1) {
          thr_reg = nk1 < bnd ? nk1 : bnd;
          cnt_reg = 0;
          if (!FLT && a.share && nk1 != kEmptyKey)
            atomicMin(a.share + qrow, (unsigned int)(nk1 >> 32));
          if (EW > 1 && nk1 != kEmptyKey) atomicMin(rowthr + erow, nk1);
        }
        __syncwarp();
      }
    };
    // Row norms (L2) are loaded one tile ahead into registers, so their global
    // load latency overlaps the previous tile's epilogue; each warp stages its
    // own copy, so no barrier spans the four warps. pf_r0 tags the tile the
    // registers hold; a mismatch (first tile, an empty item) reloads.
    constexpr int kPf = kCols / 32;
    float xn_pf[kPf];
    long long pf_r0 = -1;
    auto load_norms = [&](long long r0, long long re) {
#pragma unroll
      for (int i = 0; i < kPf; ++i) {
        const long long r = r0 + cbeg + lane + 32 * i;
        xn_pf[i] = r < re ? a.xnorms[r] : 0.0f;
      }
      pf_r0 = r0;
    };
    for (uint32_t qi = 0;; ++qi) {
      const int qs = qi % kTqQueue;
      if (!mbar_wait(&qfull[qs], (qi / kTqQueue) & 1, s_abort, &g_device_error)) break;
      const int item = s_q[qs].item;
      const ItemDesc it = s_q[qs].it;
      __syncwarp();
      if (lane == 0) mbar_arrive(&qempty[qs]);
      if (item < 0) break;
      if (tid == 0) TQT(FLT, g_tc_trace_item, qi, 2, kTrItems);
      const long long nrows = it.re > it.rb ? it.re - it.rb : 0;
      const int nT = (int)((nrows + BN - 1) / BN);
      const bool valid = erow < it.nq_item;
      long long slot = -1;
      int q = 0;
      if (valid) {
        if (a.flat) {
          q = it.a_row0 + erow;
          slot = a.direct ? q : (long long)q * a.P + it.part;
        } else {
          const int pr = a.pairs[it.a_row0 + erow];
          q = pr / a.P;
          slot = pr;
        }
      }
      float qn = 0.0f;
      if (METRIC == MF_METRIC_L2 && valid) qn = a.pair_qn ? a.pair_qn[slot] : a.qnorms[q];
      // FLT: the accumulators are s_q s_l times the dot products
      const float sc = (FLT && valid) ? a.pair_sc[slot] : 1.0f;
      const float m2s = -2.0f * sc;
      // FLT: u = qn - 2 sc acc, so u <= thr iff acc >= (qn - thr) / (2 sc)
      const float h2 = 0.5f / sc;  // exact: sc is a power of two
      for (int i = 0; i < 32 * KC; i += 32) my_lists[i + lane] = kEmptyKey;
      __syncwarp();
      unsigned long long bound = kEmptyKey;
      if (valid && a.pair_thr) bound = bound_key(a.pair_thr[slot]);
      else if (valid && a.bound) bound = bound_key(a.bound[q]);
      unsigned long long thr = bound;
      int cnt = 0;
      // the other pieces' k-th distance for this row's query, loaded one tile
      // ahead of its use
      unsigned int sh_pf = (!FLT && a.share && valid) ? __ldcg(a.share + q) : ~0u;

      for (int t = 0; t < nT; ++t, ++tt) {
        const int b = tt % NACC;
        const long long r0 = it.rb + (long long)t * BN;
        if (!FLT && a.share) {  // flat searches only (never the filter scan)
          if (sh_pf != ~0u) {
            // every row with a distance <= that bound passes, as bound_key keeps it
            const unsigned long long sk =
                (static_cast<unsigned long long>(sh_pf) << 32) | 0xffffffffull;
            if (sk < bound) bound = sk;
            if (sk < thr) thr = sk;
          }
          sh_pf = valid ? __ldcg(a.share + q) : ~0u;
        }
#ifdef MF_TC_PROFILE
        const long long p_s0 = clock64();
#endif
        if (METRIC == MF_METRIC_L2 && !FLT) {
          // row norms of this tile, shared by the four epilogue warps
          if (pf_r0 != r0) load_norms(r0, it.re);
          float* xs = xn_s + (ewarp * 2 + (tt & 1)) * BN;
#pragma unroll
          for (int i = 0; i < kPf; ++i) xs[cbeg + lane + 32 * i] = xn_pf[i];
          __syncwarp();
          // issue the next tile's loads now; they land while this tile runs
          if (t + 1 < nT) {
            load_norms(r0 + BN, it.re);
          } else {
            // the next item, if the producer has published it already
            const uint32_t nq = qi + 1;
            if (mbar_test(&qfull[nq % kTqQueue], (nq / kTqQueue) & 1)) {
              const QSlot& ns = s_q[nq % kTqQueue];
              if (ns.item >= 0 && ns.it.re > ns.it.rb) load_norms(ns.it.rb, ns.it.re);
            }
          }
        }
#ifdef MF_TC_PROFILE
        p_stage += clock64() - p_s0;
#endif
        TQL(p_wait,
            mbar_wait<FLT && kTcSpin>(&accf[b], (tt / NACC) & 1, s_abort, &g_device_error));
        if (tid == 0) TQT(FLT, g_tc_trace, tt, 3, kTrTiles);
#ifdef MF_TC_PROFILE
        ++p_tiles;
#endif
        tc_fence_after();
        if (EW > 1) {
          // the other group's best k-th key for this row bounds it too
          const unsigned long long o = *(volatile unsigned long long*)(rowthr + erow);
          if (o < thr) thr = o;
        }
        const float* xs = xn_s + (ewarp * 2 + (tt & 1)) * BN;
        // One 32-column chunk: filter, merge rows that would overflow, append.
        auto chunk = [&](uint32_t (&r)[32], int c0) {
          const long long rc = r0 + c0;
          const long long left = it.re - rc;
          const int nvalid = left >= 32 ? 32 : (left > 0 ? (int)left : 0);
          const float thr_d = thr == kEmptyKey ? __int_as_float(0x7f800000) : key_dist(thr);
#ifdef MF_TC_PROFILE
          const long long p_f0 = clock64();
#endif
          unsigned int acc;
          if (FLT) {
            // The exact form keeps a column iff RN(qn - 2 sc acc) <= thr, which
            // implies acc >= (qn - thr - ulp(thr) / 2) h2. tau lowers the
            // computed (qn - thr) h2 by 2^-22 (|qn| + |thr|) h2, more than that
            // half ulp plus the roundings of tau itself, so every such column
            // passes (a few just above thr may pass too: the merge orders them
            // by their exact key). thr = +inf gives tau = -inf: all pass.
            const float tau = (qn - thr_d) * h2 - (fabsf(qn) + fabsf(thr_d)) * h2 * 0x1p-22f;
            // Most chunks keep nothing: the chunk's largest accumulator says
            // whether any column can pass (exactly: acc >= tau for some
            // column iff their maximum is >= tau); only then is the mask built.
            const bool hit = valid && (nvalid < 32 ? nvalid > 0 : max32(r) >= tau);
            if (!__any_sync(0xffffffffu, hit)) {
#ifdef MF_TC_PROFILE
              p_filter += clock64() - p_f0;
#endif
              return;
            }
            acc = hit ? tq_accept_acc(r, tau, nvalid) : 0u;
          } else {
            acc = tq_accept<METRIC>(r, xs + c0, qn, m2s, thr_d, nvalid);
            if (!valid) acc = 0;
          }
          const unsigned int over = __ballot_sync(0xffffffffu, cnt + __popc(acc) > 32);
#ifdef MF_TC_PROFILE
          p_filter += clock64() - p_f0;
          const long long p_a0 = clock64();
          if (__any_sync(0xffffffffu, acc != 0)) ++p_nappend;
#endif
          if (over) {
            TQL(p_merge, merge_rows(over, cnt, thr, bound, q));
#ifdef MF_TC_PROFILE
            p_nmerge += __popc(over);
#endif
          }
          // The survivors' keys. FLT: u = qn - 2 sc acc (the norm is in the
          // accumulator), clamped at 0.
          auto key_of = [&](uint32_t bits, int j) {
            const float v = __uint_as_float(bits);
            const float dist = FLT ? fmaxf(fmaf(m2s, v, qn), 0.0f) + 0.0f
                               : (METRIC == MF_METRIC_L2 ? l2_from_dot(qn, xs[c0 + j], v) : -v);
            return make_key(dist, (unsigned int)(rc + j));
          };
          // A lane loops over its own set bits while every lane has few (the
          // column's value selected by a 5-level mux tree). A warp with a busy
          // lane (an open list at the start of a flat piece) takes every
          // column in turn with static register indices instead, so its cost
          // stops growing with the busiest lane's count. The filter scan keeps
          // the loop alone: its survivors are rarer, and the extra code slowed it.
          if (!FLT &&
              __reduce_max_sync(0xffffffffu, (unsigned int)__popc(acc)) > kTqSerialSurvivors) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (acc & (1u << j)) own_buf[cnt++] = key_of(r[j], j);
          } else {
            for (unsigned int m = acc; m != 0u; m &= m - 1u) {
              const int j = __ffs(m) - 1;
              own_buf[cnt++] = key_of(select32(r, j), j);
            }
          }
          __syncwarp();
#ifdef MF_TC_PROFILE
          p_append += clock64() - p_a0;
#endif
        };
        const uint32_t tb = tmem + ((uint32_t)(eq * 32) << 16) + L.acc0 + b * BN;
        if constexpr (!FLT) {
          if (a.dmat) {
            // the distance-matrix path: this row's distances of the tile,
            // stored as the top-k would key them (rows past the bank land in
            // padding columns), then the accumulator is free
#pragma unroll 1
            for (int c0 = cbeg; c0 < cend; c0 += 32) {
              uint32_t r[32];
              tmem_ld32_async(tb + c0, r);
              tmem_wait_ld(r);
              if (valid) {
                float4* dst =
                    reinterpret_cast<float4*>(a.dmat + (long long)q * a.dmat_ld + r0 + c0);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  float v[4];
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    const float x = __uint_as_float(r[4 * i + j]);
                    v[j] = METRIC == MF_METRIC_L2 ? l2_from_dot(qn, xs[c0 + 4 * i + j], x) : -x;
                  }
                  __stcs(dst + i, make_float4(v[0], v[1], v[2], v[3]));
                }
              }
            }
            tc_fence_before();
            mbar_arrive(&acce[b]);
            continue;
          }
        }
        // TMEM loads are double-buffered: chunk c+1 loads while c is filtered.
        uint32_t ra[32], rb[32];
        tmem_ld32_async(tb + cbeg, ra);
#pragma unroll 1
        for (int c0 = cbeg; c0 < cend; c0 += 64) {
          TQL(p_tld, tmem_wait_ld(ra));
          if (tid == 0 && c0 == cbeg) TQT(FLT, g_tc_trace, tt, 5, kTrTiles);
          tmem_ld32_async(tb + c0 + 32, rb);
          chunk(ra, c0);
          TQL(p_tld, tmem_wait_ld(rb));
          if (c0 + 64 < cend) tmem_ld32_async(tb + c0 + 64, ra);
          chunk(rb, c0 + 32);
          if (tid == 0 && c0 == cbeg) TQT(FLT, g_tc_trace, tt, 6, kTrTiles);
        }
        if (tid == 0) TQT(FLT, g_tc_trace, tt, 7, kTrTiles);
        tc_fence_before();
        mbar_arrive(&acce[b]);
        if (tid == 0) TQT(FLT, g_tc_trace, tt, 4, kTrTiles);
      }
      // flush the remaining candidates, then write each row's k keys
#ifdef MF_TC_PROFILE
      const long long p_o0 = clock64();
#endif
      const unsigned int pending = __ballot_sync(0xffffffffu, cnt > 0);
      if (pending) merge_rows(pending, cnt, thr, bound, q);
      if constexpr (EW > 1) {
        // The second group hands its rows' lists to the first, which merges
        // them into its own (the k smallest of both: the elementwise minimum
        // against the other list reversed is bitonic) and writes the results.
        // Both groups take the same items in the same order, so the item's
        // queue index gives the handshake's phase. Each row's shared k-th key
        // is cleared before the second group may start the next item.
        const uint32_t ph = qi & 1;
        if (eg == 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(wgdone);
          if (!mbar_wait(wgfree, ph, s_abort, &g_device_error)) break;
          continue;
        }
        if (!mbar_wait(wgdone, ph, s_abort, &g_device_error)) break;
        const unsigned long long* other = lists + (size_t)kTqM * KC + (size_t)(eq * 32) * KC;
        for (int r = 0; r < 32; r += 2) {
          unsigned long long x[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const unsigned long long e0 = my_lists[(r + i) * KC + lane];
            const unsigned long long e1 = other[(r + i) * KC + 31 - lane];
            x[i] = e0 < e1 ? e0 : e1;
          }
          warp_bitonic_clean32_n<2>(x, lane);
#pragma unroll
          for (int i = 0; i < 2; ++i) my_lists[(r + i) * KC + lane] = lane < k ? x[i] : kEmptyKey;
        }
        rowthr[erow] = kEmptyKey;
        __syncwarp();
        if (lane == 0) mbar_arrive(wgfree);
      }
      if (FLT) {
        // the kept slots of each row (a sorted prefix) and their count; rows
        // that kept none write nothing (their counts start at 0)
        const unsigned int some =
            __ballot_sync(0xffffffffu, slot >= 0 && my_lists[lane * KC] != kEmptyKey);
        for (unsigned int mq = some; mq != 0u; mq &= mq - 1u) {
          const int qq = __ffs(mq) - 1;
          const long long sq = __shfl_sync(0xffffffffu, slot, qq);
          const unsigned long long key = lane < k ? my_lists[qq * KC + lane] : kEmptyKey;
          const unsigned int m = __ballot_sync(0xffffffffu, key != kEmptyKey);
          if (lane == 0) a.pair_cnt[sq] = __popc(m);
          if (key != kEmptyKey) {
            a.out_d[sq * k + lane] = key_dist(key);
            a.out_l[sq * k + lane] = (long long)key_index(key);
          }
        }
      }
      // the warp's 32 rows x k results, one per lane per step: the k steps are
      // independent, so their id lookups overlap
      for (int e = lane; e < ((FLT || a.dmat) ? 0 : 32 * k); e += 32) {
        const int qq = e / k;
        const int kk = e - qq * k;
        const long long sq = __shfl_sync(0xffffffffu, slot, qq);
        if (sq >= 0) {
          const unsigned long long key = my_lists[qq * KC + kk];
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
          a.out_d[sq * k + kk] = dv;
          a.out_l[sq * k + kk] = lv;
        }
      }
      __syncwarp();
#ifdef MF_TC_PROFILE
      p_out += clock64() - p_o0;
#endif
      if (tid == 0) TQT(FLT, g_tc_trace_item, qi, 3, kTrItems);
    }
#ifdef MF_TC_PROFILE
    p_loop = clock64() - p_start;
    if (tid == 0) {
      atomicAdd(&g_tc_prof[3], (unsigned long long)p_wait);
      atomicAdd(&g_tc_prof[4], (unsigned long long)p_loop);
      atomicAdd(&g_tc_prof[5], (unsigned long long)p_tiles);
      atomicAdd(&g_tc_prof[7], (unsigned long long)p_merge);
      atomicAdd(&g_tc_prof[11], (unsigned long long)p_nmerge);
      atomicAdd(&g_tc_prof[12], (unsigned long long)p_out);
      atomicAdd(&g_tc_prof[6], (unsigned long long)p_stage);
      atomicAdd(&g_tc_prof[9], (unsigned long long)p_filter);
      atomicAdd(&g_tc_prof[10], (unsigned long long)p_append);
      atomicAdd(&g_tc_prof[14], (unsigned long long)p_tld);
      atomicAdd(&g_tc_prof[15], (unsigned long long)p_nappend);
    }
#endif
  }

  // ---- teardown: stages in flight land and MMAs finish before TMEM is freed
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 4 * 32) {
    // the last use of each stage: its loads have landed once that phase is
    // complete (earlier uses were complete before their stage was reissued)
    int dummy = 0;
    const uint32_t issued = s_seq[1];
    for (uint32_t seq = issued > (uint32_t)SA ? issued - SA : 0; seq < issued; ++seq)
      mbar_wait(&full[seq % SA], (seq / SA) & 1, &dummy, &g_device_error);
  }
  __syncthreads();
  if (warp == 5) {
    if (lane == 0) {
      int dummy = 0;
      mbar_wait(mdone, 0, &dummy, &g_device_error);
    }
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTqTmemCols);
  }
#ifdef MF_TC_PROFILE
  if (tid == 0) atomicAdd(&g_tc_prof[13], (unsigned long long)(clock64() - _tk));
#endif
}

// ------------------------------------------------------------------ host
typedef void (*TqFn)(const ScanArgs, const TqMaps, const TqLayout);

template <int METRIC>
TqFn pick_tq(const TqLayout& l, bool conv, int kcap) {
  if (kcap > kTqK) {  // 64-row tiles, query tile in tensor memory (d <= 128)
    if (!l.atm || l.BN != 64) return nullptr;
    return conv ? tq_scan_kernel<METRIC, 64, true, true, false, kTqKBig>
                : tq_scan_kernel<METRIC, 64, true, false, false, kTqKBig>;
  }
  if (l.atm)
    return conv ? tq_scan_kernel<METRIC, 128, true, true> : tq_scan_kernel<METRIC, 128, true, false>;
  return l.BN == 256 ? tq_scan_kernel<METRIC, 256, false, false>
                     : tq_scan_kernel<METRIC, 128, false, false>;
}

int tq_kcap(int k) { return k <= kTqK ? kTqK : (k <= kTqKBig ? kTqKBig : 0); }

int g_engine = 0;  // 0 auto, 1 SIMT only, 2 tensor cores where eligible, 3 = 2 with streamed queries
int g_filter_groups = 2;  // epilogue warpgroups of the filter scan (1 or 2)

// With d <= 128 the query tile (hi and lo) lives in tensor memory next to two
// accumulator buffers, and shared memory holds only row stages: the deepest
// ring that fits. Otherwise the widest tile (BN rows) and deepest ring with
// the query tile streamed beside the rows.
bool tq_choose(int d, int kcap, TqLayout* out) {
  const int kb32 = (d + 31) / 32 * 32;
  if (kcap > kTqK) {
    // 128-key lists (128 KB for the tile's rows): 64-row tiles, query tile in
    // tensor memory, the deepest ring that fits
    if (g_engine == 3 || kb32 > kTqMaxDAtm) return false;
    for (int sa = 5; sa >= 2; --sa) {
      TqLayout l = tq_layout(d, kcap, 64, sa, true);
      if (l.total <= (size_t)kTqMaxSmem) {
        *out = l;
        return true;
      }
    }
    return false;
  }
  if (g_engine != 3 && kb32 <= kTqMaxDAtm && kTqTmemCols - 2 * kb32 >= 2 * 128) {
    for (int sa = 5; sa >= 2; --sa) {
      TqLayout l = tq_layout(d, kcap, 128, sa, true);
      if (l.total <= (size_t)kTqMaxSmem) {
        *out = l;
        return true;
      }
    }
  }
  const int cands[4][2] = {{256, 3}, {256, 2}, {128, 3}, {128, 2}};
  for (auto& c : cands) {
    TqLayout l = tq_layout(d, kcap, c[0], c[1], false);
    if (l.total <= (size_t)kTqMaxSmem) {
      *out = l;
      return true;
    }
  }
  return false;
}

// The filter scan (fp16, 64 <= d <= 128 with rows of a multiple of 16 bytes):
// the query tile in tensor memory and the deepest ring of 16 KB row stages
// that fits. (d >= 64: no tile box wider than the rows.)
// Build-time caps on the filter scan's ring depth and accumulator buffers
// (tuning builds; the defaults take what fits).
#ifndef MF_FLT_MAX_SA
#define MF_FLT_MAX_SA 8
#endif
#ifndef MF_FLT_MAX_NACC
#define MF_FLT_MAX_NACC kTqMaxAcc
#endif

bool tq_choose_bf(int d, TqLayout* out) {
  if (d < 64 || d > kTqMaxDAtm || d % 8 != 0) return false;
  // two epilogue warpgroups where their lists and buffers leave room for a
  // ring of at least two stages (g_filter_groups = 1 forces one)
  for (int ew = g_filter_groups; ew >= 1; --ew) {
    // an even ring: stage s then always serves tiles of one MMA issuer
    for (int sa = MF_FLT_MAX_SA & ~1; sa >= 2; sa -= 2) {
      TqLayout l = tq_layout(d, kTqK, 128, sa, true, true, ew);
      if (l.nacc > MF_FLT_MAX_NACC) l.nacc = MF_FLT_MAX_NACC;
      if (l.total <= (size_t)kTqMaxSmem) {
        *out = l;
        return true;
      }
    }
  }
  return false;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_tc_mu;
int g_tc_attr[64][2][8];  // dynamic smem set per (device, metric, variant)

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

int make_map(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, const float* p, int d,
             int64_t rows, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)d * 4};
  cuuint32_t box[2] = {32, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MF_CHECK(r == CUDA_SUCCESS, MF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MF_OK;
}

// fp16 rows of d elements (d a multiple of 8: 16-byte row pitch), tiles of
// 64 x box_rows (128-byte inner box, 128-byte swizzle).
int make_map_f16(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, const void* p, int d,
                  int64_t rows, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)d, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)d * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MF_CHECK(r == CUDA_SUCCESS, MF_ERR_CUDA, "cuTensorMapEncodeTiled (fp16) failed (%d)", (int)r);
  return MF_OK;
}

// The filter bank's 16-element fp16 norm extensions: rows of 32 bytes, tiles
// of 16 x box_rows (32-byte inner box, 32-byte swizzle).
int make_map_rn16(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, const void* p,
                  int64_t rows, int box_rows) {
  cuuint64_t dims[2] = {16, (cuuint64_t)rows};
  cuuint64_t strides[1] = {32};
  cuuint32_t box[2] = {16, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(p), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  MF_CHECK(r == CUDA_SUCCESS, MF_ERR_CUDA, "cuTensorMapEncodeTiled (norm extensions) failed (%d)",
           (int)r);
  return MF_OK;
}

__global__ void tf32_residual_kernel(const float4* __restrict__ x, int64_t n4, float4* lo) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 v = x[i];
  float4 h, l;
  split_tf32(v.x, h.x, l.x);
  split_tf32(v.y, h.y, l.y);
  split_tf32(v.z, h.z, l.z);
  split_tf32(v.w, h.w, l.w);
  lo[i] = l;
}

// Gathered query rows for IVF items: row p of (g_hi, g_lo) = query pairs[p] / P.
__global__ void gather_queries_kernel(const float* __restrict__ xq, int d,
                                      const int* __restrict__ pairs,
                                      const int* __restrict__ n_pairs, int P, float* g_hi,
                                      float* g_lo) {
  const int p = blockIdx.x;
  if (p >= *n_pairs) return;
  const int q = pairs[p] / P;
  const float4* src = reinterpret_cast<const float4*>(xq + (int64_t)q * d);
  float4* dh = reinterpret_cast<float4*>(g_hi + (int64_t)p * d);
  float4* dl = reinterpret_cast<float4*>(g_lo + (int64_t)p * d);
  for (int j = threadIdx.x; j < (d >> 2); j += blockDim.x) {
    const float4 v = src[j];
    float4 h, l;
    split_tf32(v.x, h.x, l.x);
    split_tf32(v.y, h.y, l.y);
    split_tf32(v.z, h.z, l.z);
    split_tf32(v.w, h.w, l.w);
    dh[j] = v;
    dl[j] = l;
  }
}

// Accumulation probe (a diagnostic, not on the search path): out (128 x 128)
// = A (128 x d) . B (128 x d)^T in the filter pass's instruction form. A
// (fp16) sits in tensor memory, written by tcgen05.st two elements per
// column; B (fp16) arrives by TMA in the 128-byte swizzled K-major layout,
// K-blocks of 64; one tcgen05.mma kind::f16 per 16 of K accumulates in fp32
// in tensor memory. One CTA of 128 threads; thread t owns row t of A and of
// the result. Every wait is bounded.
__global__ void __launch_bounds__(128, 1)
    tc_f16_probe_kernel(const __grid_constant__ CUtensorMap bmap, const uint32_t* __restrict__ a,
                        int d, float* __restrict__ out) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int KB = (d + 63) / 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + size_t(KB) * kTqM * 128);
  uint64_t* done = full + 1;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(done + 1);
  int* s_abort = reinterpret_cast<int*>(s_tmem + 1);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  if (warp == 0) {
    tmem_alloc(s_tmem, 256);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(full, 1);
    mbar_init(done, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
  const int words = d / 2;  // 32-bit words (fp16 pairs) per row
  const uint32_t* arow = a + (size_t)tid * words;
  for (int c = 0; c < KB; ++c) {
    uint32_t pk[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const int w = c * 32 + i;
      pk[i] = w < words ? arow[w] : 0u;
    }
    tmem_st32(lane_base + c * 32, pk);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t acc = tmem + 128;  // accumulator columns [128, 256)
  if (tid == 0) {
    mbar_arrive_expect_tx(full, (uint32_t)(KB * kTqM * 128));
    for (int kb = 0; kb < KB; ++kb) tma_load_2d(base + size_t(kb) * kTqM * 128, &bmap, kb * 64, 0, full);
    if (mbar_wait(full, 0, s_abort, &g_device_error)) {
      tc_fence_after();
      const uint32_t st = smem_u32(base);
      constexpr uint32_t idesc = idesc_f16(kTqM, 128);
      for (int kb = 0; kb < KB; ++kb)
        for (int kk = 0; kk < 4; ++kk)
          mma_f16_ts(acc, tmem + kb * 32 + kk * 8,
                     desc_k_sw128(st + (uint32_t)(kb * kTqM * 128) + kk * 32), idesc,
                     !(kb == 0 && kk == 0));
      mma_commit(done);
    }
  }
  __syncthreads();
  const bool ok = mbar_wait(done, 0, s_abort, &g_device_error);
  tc_fence_after();
  if (ok) {
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tmem_ld32(lane_base + 128 + c * 32, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) out[(size_t)tid * 128 + c * 32 + i] = v[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

int launch_f16_probe_tc(const void* a, const void* b, int d, float* out, cudaStream_t stream) {
  MF_CHECK(d >= 64 && d <= kTqMaxDAtm && d % 8 == 0, MF_ERR_INVALID_ARGS,
           "tensor-core probe: d=%d (64 <= d <= 128, a multiple of 8)", d);
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  MF_TRY(encoder(&enc));
  CUtensorMap map;
  MF_TRY(make_map_f16(enc, &map, b, d, kTqM, kTqM));
  const int KB = (d + 63) / 64;
  const size_t smem = size_t(KB) * kTqM * 128 + 64 + 1024;
  tc_f16_probe_kernel<<<1, 128, smem, stream>>>(map, reinterpret_cast<const uint32_t*>(a), d,
                                                out);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

void set_scan_engine(int e) { g_engine = e; }
void set_filter_groups(int g) { g_filter_groups = g == 1 ? 1 : 2; }
int scan_engine() { return g_engine; }

int tc_group() { return kTqM; }

bool tc_eligible(int metric, int d, int k, int64_t xb_rows) {
  if (g_engine == 1) return false;
  if (metric != MF_METRIC_L2 && metric != MF_METRIC_INNER_PRODUCT) return false;
  if (d < 32 || d > kTqMaxD || d % 4 != 0) return false;
  if (xb_rows < 256) return false;
  const int kcap = tq_kcap(k);
  if (kcap == 0) return false;
  TqLayout l;
  return tq_choose(d, kcap, &l);
}

bool tc_raw_queries(int d, int k) {
  TqLayout l;
  const int kcap = tq_kcap(k);
  return kcap != 0 && tq_choose(d, kcap, &l) && l.atm;
}

int launch_tf32_residual(const float* x, int64_t n, int d, float* lo, cudaStream_t stream) {
  const int64_t n4 = n * (int64_t)d / 4;
  if (n4 <= 0) return MF_OK;
  tf32_residual_kernel<<<(unsigned int)ceil_div(n4, 256), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(x), n4, reinterpret_cast<float4*>(lo));
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_gather_queries(const float* xq, int d, const int* pairs, const int* n_pairs,
                          int64_t max_pairs, int P, float* g_hi, float* g_lo,
                          cudaStream_t stream) {
  if (max_pairs <= 0) return MF_OK;
  gather_queries_kernel<<<(unsigned int)max_pairs, 64, 0, stream>>>(xq, d, pairs, n_pairs, P,
                                                                    g_hi, g_lo);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

int launch_tc_scan(const ScanArgs& a, int metric, const float* a_lo, int64_t a_rows,
                   const float* b_lo, int64_t b_rows, int64_t total_items, int device,
                   cudaStream_t stream) {
  const int kcap = tq_kcap(a.k);
  TqLayout lay;
  MF_CHECK(kcap != 0 && tq_choose(a.d, kcap, &lay), MF_ERR_INVALID_ARGS,
           "tensor-core scan does not fit (d=%d k=%d)", a.d, a.k);
  const bool conv = lay.atm && b_lo == nullptr;  // derive the rows' residuals in the kernel
  TqFn fn = metric == MF_METRIC_L2 ? pick_tq<MF_METRIC_L2>(lay, conv, kcap)
                                   : pick_tq<MF_METRIC_INNER_PRODUCT>(lay, conv, kcap);
  MF_CHECK(fn != nullptr, MF_ERR_METRIC, "metric %d has no tensor-core scan", metric);
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  MF_TRY(encoder(&enc));
  TqMaps maps;
  memset(&maps, 0, sizeof(maps));
  if (!lay.atm) {  // streamed query tile: a.xq / a_lo hold one row per A row
    MF_TRY(make_map(enc, &maps.a_hi, a.xq, a.d, a_rows, kTqM));
    MF_TRY(make_map(enc, &maps.a_lo, a_lo, a.d, a_rows, kTqM));
  }
  MF_TRY(make_map(enc, &maps.b_hi, a.xb, a.d, b_rows, lay.BN));
  if (!conv) {
    MF_CHECK(b_lo != nullptr, MF_ERR_INVALID_ARGS, "tensor-core scan needs the rows' residuals");
    MF_TRY(make_map(enc, &maps.b_lo, b_lo, a.d, b_rows, lay.BN));
  }
  {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    const int mi = metric == MF_METRIC_L2 ? 0 : 1;
    const int bi = kcap > kTqK ? (conv ? 6 : 5)
                               : (lay.atm ? (conv ? 3 : 2) : (lay.BN == 256 ? 1 : 0));
    if (device < 0 || device >= 64 || g_tc_attr[device][mi][bi] < (int)lay.total) {
      MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.total));
      if (device >= 0 && device < 64) g_tc_attr[device][mi][bi] = (int)lay.total;
    }
  }
  if (total_items <= 0) return MF_OK;
  MF_CHECK(a.counter != nullptr, MF_ERR_INVALID_ARGS, "tensor-core scan needs a work counter");
  MF_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(int), stream));
  long long grid = num_sms(device);
  if (grid > total_items) grid = total_items;
  ScopedTiming tm(a.flat ? "scan_topk_flat" : (a.max_rows > 0 ? "scan_topk_ivf_bound" : "scan_topk_ivf"), stream);
  fn<<<(unsigned int)grid, lay.atm ? kTqThreadsAtm : kTqThreads, lay.total, stream>>>(a, maps, lay);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

bool tc_filter_eligible(int d) {
  if (g_engine == 1) return false;
  TqLayout l;
  return tq_choose_bf(d, &l);
}

int filter_slots() { return kTqK; }

int launch_tc_filter(const ScanArgs& a, int64_t b_rows, int64_t total_items, int device,
                     cudaStream_t stream) {
  TqLayout lay;
  MF_CHECK(a.k >= 1 && a.k <= kTqK && tq_choose_bf(a.d, &lay), MF_ERR_INVALID_ARGS,
           "filter scan does not fit (d=%d k=%d)", a.d, a.k);
  MF_CHECK(!a.flat && a.pair_qn && a.pair_thr && a.pair_sq && a.pair_sc && a.pair_cnt &&
               a.pair_ae && a.xrn16 && a.centroids && a.items && a.item_total,
           MF_ERR_INVALID_ARGS, "filter scan needs IVF items and its per-pair arrays");
  TqFn fn = lay.ew == 2 ? tq_scan_kernel<MF_METRIC_L2, 128, true, false, true, kTqK, 2>
                        : tq_scan_kernel<MF_METRIC_L2, 128, true, false, true, kTqK, 1>;
  const int slot = lay.ew == 2 ? 7 : 4;
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  MF_TRY(encoder(&enc));
  TqMaps maps;
  memset(&maps, 0, sizeof(maps));
  MF_TRY(make_map_f16(enc, &maps.b_hi, a.xb, a.d, b_rows, lay.BN));
  MF_TRY(make_map_rn16(enc, &maps.b_lo, a.xrn16, b_rows, lay.BN));
  {
    std::lock_guard<std::mutex> lk(g_tc_mu);
    if (device < 0 || device >= 64 || g_tc_attr[device][0][slot] < (int)lay.total) {
      MF_CUDA(cudaFuncSetAttribute(reinterpret_cast<const void*>(fn),
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.total));
      if (device >= 0 && device < 64) g_tc_attr[device][0][slot] = (int)lay.total;
    }
  }
  if (total_items <= 0) return MF_OK;
  MF_CHECK(a.counter != nullptr, MF_ERR_INVALID_ARGS, "filter scan needs a work counter");
  MF_CUDA(cudaMemsetAsync(a.counter, 0, sizeof(int), stream));
  long long grid = num_sms(device);
  if (grid > total_items) grid = total_items;
  ScopedTiming tm("scan_topk_ivf_filter", stream);
  // + the second MMA issuer's warp
  fn<<<(unsigned int)grid, kTqThreadsAtm + (lay.ew - 1) * kTqEpiThreads + 32, lay.total, stream>>>(
      a, maps, lay);
  MF_LAUNCH_CHECK();
  return MF_OK;
}

#ifdef MF_TC_STAMPS
extern "C" MF_API int mf_tc_trace_read(long long* tiles, long long* items, int reset) {
  MF_CUDA(cudaMemcpyFromSymbol(tiles, g_tc_trace, sizeof(g_tc_trace)));
  MF_CUDA(cudaMemcpyFromSymbol(items, g_tc_trace_item, sizeof(g_tc_trace_item)));
  if (reset) {
    void* p = nullptr;
    MF_CUDA(cudaGetSymbolAddress(&p, g_tc_trace));
    MF_CUDA(cudaMemset(p, 0, sizeof(g_tc_trace)));
    MF_CUDA(cudaGetSymbolAddress(&p, g_tc_trace_item));
    MF_CUDA(cudaMemset(p, 0, sizeof(g_tc_trace_item)));
  }
  return MF_OK;
}
#endif
#ifdef MF_TC_PROFILE
extern "C" MF_API int mf_tc_profile_read(unsigned long long* out16, int reset) {
  MF_CUDA(cudaMemcpyFromSymbol(out16, g_tc_prof, 20 * sizeof(unsigned long long)));
  if (reset) {
    unsigned long long z[20] = {0};
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
