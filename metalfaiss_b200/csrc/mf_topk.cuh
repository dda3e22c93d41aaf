// Warp-cooperative top-k selection over 64-bit keys (see mf_common.cuh).
//
// One warp owns one query's state: a sorted list of the k best keys in shared
// memory and a 32-entry candidate buffer. A batch of 32 candidates (one per
// lane) is filtered against the k-th best key; survivors are appended to the
// buffer. A full buffer is sorted across the lanes (bitonic network on
// shuffles) and merged into the list in place: every element's new position is
// its old position plus its rank in the other sequence, so all positions are
// computed before any write. The design follows the register/shared-memory
// k-selection of Johnson, Douze and Jegou, "Billion-scale similarity search with
// GPUs" (2017), which the reference's top-k kernel stubs cite
// (python/metalfaiss/faissmlx/kernels/topk_kernels.py:4,16-31).
#pragma once

#include "mf_common.cuh"

namespace mf {

// Ascending bitonic sort of 32 keys, one per lane.
__device__ __forceinline__ unsigned long long warp_sort32(unsigned long long c, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      unsigned long long o = __shfl_xor_sync(0xffffffffu, c, stride);
      bool up = (lane & size) == 0;
      bool low = (lane & stride) == 0;
      c = (low == up) ? (c < o ? c : o) : (c < o ? o : c);
    }
  }
  return c;
}

// N independent ascending bitonic sorts of 32 keys (one per lane each), with
// their shuffle stages interleaved so the latencies overlap.
template <int N>
__device__ __forceinline__ void warp_sort32_n(unsigned long long (&c)[N], int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const bool up = (lane & size) == 0;
      const bool low = (lane & stride) == 0;
      unsigned long long o[N];
#pragma unroll
      for (int i = 0; i < N; ++i) o[i] = __shfl_xor_sync(0xffffffffu, c[i], stride);
#pragma unroll
      for (int i = 0; i < N; ++i)
        c[i] = (low == up) ? (c[i] < o[i] ? c[i] : o[i]) : (c[i] < o[i] ? o[i] : c[i]);
    }
  }
}

// Sorts N bitonic 32-key sequences ascending (half-cleaners, strides 16..1).
template <int N>
__device__ __forceinline__ void warp_bitonic_clean32_n(unsigned long long (&x)[N], int lane) {
#pragma unroll
  for (int st = 16; st > 0; st >>= 1) {
    unsigned long long o[N];
#pragma unroll
    for (int i = 0; i < N; ++i) o[i] = __shfl_xor_sync(0xffffffffu, x[i], st);
#pragma unroll
    for (int i = 0; i < N; ++i)
      x[i] = (lane & st) ? (x[i] > o[i] ? x[i] : o[i]) : (x[i] < o[i] ? x[i] : o[i]);
  }
}

// Number of lanes whose (sorted, ascending) key is < e.
// Binary search over the 32 lane-distributed keys; every lane runs the same
// shuffles but searches for its own e. The five halving steps resolve 0..31;
// the last lane's key decides 32.
__device__ __forceinline__ int warp_rank_below(unsigned long long sorted, unsigned long long e) {
  unsigned long long last = __shfl_sync(0xffffffffu, sorted, 31);
  int base = 0;
#pragma unroll
  for (int step = 16; step > 0; step >>= 1) {
    unsigned long long probe = __shfl_sync(0xffffffffu, sorted, base + step - 1);
    if (probe < e) base += step;
  }
  if (base == 31 && last < e) base = 32;
  return base;
}

// Sorts the nbuf (<= 32) buffered keys and merges them into the sorted list
// of k keys; returns the new k-th key. Out of line: it is rare on the hot path
// and keeping it out of the callers keeps their code small.
template <int KCAP>
__device__ __noinline__ unsigned long long merge_into_list(unsigned long long* list,
                                                          const unsigned long long* buf, int nbuf,
                                                          int k, int lane) {
  __syncwarp();
  unsigned long long c = (lane < nbuf) ? buf[lane] : kEmptyKey;
  c = warp_sort32(c, lane);
  constexpr int PER = (KCAP + 31) / 32;
  unsigned long long e[PER];
  int np[PER];
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    int i = lane + 32 * p;
    e[p] = (i < k) ? list[i] : kEmptyKey;
    int r = warp_rank_below(c, e[p]);
    np[p] = i + r;
  }
  int cpos = 1 << 30;
  if (lane < nbuf) {
    int lo = 0, hi = k;
    while (lo < hi) {
      int mid = (lo + hi) >> 1;
      if (list[mid] < c) lo = mid + 1; else hi = mid;
    }
    cpos = lane + lo;
  }
  __syncwarp();
#pragma unroll
  for (int p = 0; p < PER; ++p) {
    int i = lane + 32 * p;
    if (i < k && np[p] < k) list[np[p]] = e[p];
  }
  if (cpos < k) list[cpos] = c;
  __syncwarp();
  return list[k - 1];
}

// p[0..15] per lane -> the sum over the 32 lanes of p[i] in lanes 2i, 2i+1:
// a butterfly that halves the live values at each of its five steps.
__device__ __forceinline__ float warp_transpose_reduce16(float (&p)[16], int lane) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool hi = lane & 16;
    const float send = hi ? p[i] : p[i + 8];
    const float keep = hi ? p[i + 8] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 8;
    const float send = hi ? p[i] : p[i + 4];
    const float keep = hi ? p[i + 4] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 4;
    const float send = hi ? p[i] : p[i + 2];
    const float keep = hi ? p[i + 2] : p[i];
    p[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const bool hi = lane & 2;
    const float send = hi ? p[0] : p[1];
    const float keep = hi ? p[1] : p[0];
    p[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return p[0] + __shfl_xor_sync(0xffffffffu, p[0], 1);
}

// Per-query state held by the owning warp. The list lives in shared memory
// (`list`, capacity >= k); nbuf and thr are warp-uniform registers.
template <int KCAP>
struct WarpTopK {
  unsigned long long* list;  // KCAP keys, ascending; first k meaningful
  unsigned long long* buf;   // 32 keys
  int nbuf;
  unsigned long long thr;    // min(list[k-1], bound)
  unsigned long long bound;  // a key known to be no better than the final k-th

  __device__ __forceinline__ void init(unsigned long long* l, unsigned long long* b, int k,
                                       int lane, unsigned long long bnd = kEmptyKey) {
    list = l;
    buf = b;
    for (int i = lane; i < k; i += 32) list[i] = kEmptyKey;
    nbuf = 0;
    bound = bnd;
    thr = bnd;
    __syncwarp();
  }

  __device__ __forceinline__ void flush(int k, int lane) {
    if (nbuf == 0) return;
    const unsigned long long t = merge_into_list<KCAP>(list, buf, nbuf, k, lane);
    thr = t < bound ? t : bound;
    nbuf = 0;
  }

  // Offers one candidate per lane (kEmptyKey = no candidate).
  __device__ __forceinline__ void offer(unsigned long long key, int k, int lane) {
    bool pass = key < thr;
    unsigned int m = __ballot_sync(0xffffffffu, pass);
    if (m == 0u) return;
    int n = __popc(m);
    if (nbuf + n > 32) {
      flush(k, lane);
      pass = key < thr;
      m = __ballot_sync(0xffffffffu, pass);
      if (m == 0u) return;
      n = __popc(m);
    }
    if (pass) buf[nbuf + __popc(m & lanemask_lt())] = key;
    nbuf += n;
  }

  // Offers four candidates per lane; one warp vote skips the common case where
  // none of the 128 beats the current k-th best.
  __device__ __forceinline__ void offer4(const unsigned long long (&key)[4], int k, int lane) {
    const bool any = (key[0] < thr) | (key[1] < thr) | (key[2] < thr) | (key[3] < thr);
    if (!__any_sync(0xffffffffu, any)) return;
#pragma unroll
    for (int i = 0; i < 4; ++i) offer(key[i], k, lane);
  }
};

}  // namespace mf
