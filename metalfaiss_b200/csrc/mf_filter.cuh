// IVF filter search (L2): fp16 tensor-core pass + exact fp32 refinement
// (mf_filter.cu). The bank side is built once per add; the search side runs
// per batch between the bound pass and the output.
#pragma once

#include "mf_common.cuh"

namespace mf {

// Slots the filter scan keeps per pair for a top-k: 2k within [16, 32].
int filter_slots_for(int k);

// Per list row r of list l (rows [offsets[l], offsets[l+1]) of xb, d floats
// each, d a multiple of 8): h[r] = fp16(s_l (xb[r] - cents[l])) (to nearest),
// rn[r] = |xb[r] - cents[l]|^2 in fp32; per list, stats[4l..4l+3] = (R_l, an
// upper bound on the rows' residual norms; XN_l, the largest xnorms of the
// list; s_l, the list's power-of-two scale; beta_l, the power of two of the
// norm extension); R_l = XN_l = 0 for an empty list; rn16[r] = the row's
// 16-element fp16 norm extension [hi, lo, 0, ...] of beta_l rn[r] (32 bytes).
int launch_filter_bank(int nlist, int d, const int64_t* offsets, const float* xb,
                       const float* xnorms, const float* cents, void* h, float* rn, float* stats,
                       void* rn16, cudaStream_t stream);

// Per (query, probe) pair s = q*P + p of list l = probes[s] (outputs, nq*P each).
struct FilterPairs {
  float* qn;   // |q - c_l|^2 + e: the scan's query norm (e: the pair's error bound)
  float* thr;  // bound[q] + 2e: the scan's pre-filter
  float* e;
  float* sq;   // the query's power-of-two scale s_q
  float* sc;   // 1 / (s_q s_l)
  float* ae;   // -s_q s_l / (2 beta_l): the query row's norm-extension element
  int* cnt;    // kept slots: 0 here, then written by the scan
};
int launch_filter_pairs(const float* xq, const float* qnorms, int64_t nq, int P, int d,
                        const int64_t* probes, const int64_t* offsets, int nlist,
                        const float* cents, const float* stats, const float* bound,
                        const FilterPairs& fp, cudaStream_t stream);

struct RefineArgs {
  const float* xq;       // (nq, d)
  const float* qnorms;   // (nq)
  int64_t nq;
  int d;
  int P;
  int k;
  int slots;             // partial slots per pair
  const float* pd;       // (nq, P, slots) upper bounds u, ascending; cnt[s] of them kept
  const int64_t* pl;     // (nq, P, slots) row positions
  const int* cnt;        // (nq, P)
  const float* pair_e;   // (nq, P)
  const float* bound;    // (nq)
  const int64_t* probes; // (nq, P)
  const int64_t* offsets;
  const float* xb;       // rows (fp32)
  const float* xnorms;   // |x|^2
  const int64_t* ids;    // row -> id (null: the row position)
  float* D;              // (nq, k)
  int64_t* I;
};
// One warp per query: exact distances of the rows the upper bounds cannot
// exclude, exact rescans of the lists whose kept slots cannot prove it, and
// the top-k by (distance, row).
int launch_filter_refine(const RefineArgs& f, cudaStream_t stream);

// Lists rescanned by the refinement since the last reset (a statistic).
int read_filter_rescans(unsigned long long* out, bool reset);

}  // namespace mf
