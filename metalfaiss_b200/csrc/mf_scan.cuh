// Slab scan: the one SIMT kernel family behind flat kNN, the IVF list scan,
// the coarse quantizer, k-means assignment and both range-search passes.
//
// A work item is (a set of <= 32 queries, a contiguous slab of database rows).
// Flat search: items are (query tile, row split) over the whole database.
// IVF search: items are (inverted list, group of <= 32 queries probing it),
// i.e. the scan is list-major: each list slab is streamed from HBM once per
// group of queries that probe it instead of once per query.
#pragma once

#include "mf_common.cuh"

namespace mf {

constexpr int kScanThreads = 256;  // 8 warps
constexpr int kScanTQ = 32;        // queries per item (4 per warp)
constexpr int kScanTR = 128;       // rows per tile (4 per lane)
constexpr int kScanDC = 32;        // d-chunk staged per pipeline stage
constexpr int kScanXS = kScanDC + 4;  // padded smem row stride (floats): conflict-free LDS.128
constexpr int kScanStages = 4;  // cp.async ring depth: enough bytes in flight per SM to cover HBM latency

enum ScanEpilogue { kEpiTopK = 0, kEpiCount = 1, kEpiFill = 2 };

struct ScanArgs {
  const float* xq;        // (nq, d)
  const float* qnorms;    // (nq), L2 only
  const float* xb;        // (rows, d)
  const float* xnorms;    // (rows), L2 only
  const int64_t* ids;     // (rows) or null: labels are row positions
  int d;
  int k;
  int64_t nq;
  int P;                  // parts per query: row splits (flat) or nprobe (IVF)
  // flat items
  int flat;               // 1: items are (query tile, split); 0: IVF items
  int nqt;
  int64_t nb;
  int64_t rows_per_split;
  // flat on tensor cores: CTA c scans tiles [c chunk_tiles, (c+1) chunk_tiles)
  // of the (query tile x 128-row tile) space; the piece of query tile q in
  // chunk c writes partial slot c - (q tiles_per_qt) / chunk_tiles
  int64_t chunk_tiles;
  int64_t tiles_per_qt;
  // flat on tensor cores, a query tile cut into pieces: per query, the
  // smallest k-th distance any piece has reached so far (order-preserving
  // bits, all ones: none yet). Each piece publishes its own with atomicMin
  // and filters by the others': any piece's k-th distance bounds the final
  // k-th distance from above. Null: no sharing.
  unsigned int* share;
  // IVF items
  const int2* items;      // (list, group)
  const int* item_total;  // device scalar
  int group;              // queries per group the items were cut into (0: the kernel's own)
  const int64_t* list_offsets;  // (nlist+1) rows of xb
  const int* pair_offsets;      // (nlist+1) into pairs
  const int* pairs;             // q*P + slot, grouped by list
  // persistent work counter (zeroed before launch)
  int* counter;
  // top-k outputs: slot s = q*P + part (or q when direct) → [s*k, s*k+k)
  float* out_d;
  int64_t* out_l;
  int direct;
  // IVF second phase: bound[q] (a k-th distance over part of query q's nearest
  // list, an upper bound on its final k-th distance) filters every candidate;
  // null = no bound.
  const float* bound;
  // IVF items scan at most max_rows rows of their list (0 = the whole list).
  int64_t max_rows;
  // IVF filter scan (fp16 tensor cores, mf_filter.cu), per (query, probe)
  // pair s = q*P + p: pair_qn[s] stands in for the query norm (the query's
  // squared distance to the list's centroid plus the pair's error bound) and
  // pair_thr[s] for the bound; the A operand is the query minus its list's
  // centroid (centroids, rows of d floats) and xb holds the rows' fp16
  // residuals against that centroid.
  const float* pair_qn;
  const float* pair_thr;
  const float* centroids;
  // the filter scan's operands are scaled by powers of two: the query by
  // pair_sq[s], the rows by their list's scale; pair_sc[s] = 1 / (both).
  // Each pair's kept slots are a sorted prefix of its k; pair_cnt[s] = their count.
  const float* pair_sq;
  const float* pair_sc;
  int* pair_cnt;
  // the tensor-core filter pass folds the rows' residual norms into its
  // accumulator: xrn16 holds each row's 16-element fp16 extension (32 bytes:
  // [hi, lo, 0, ...] of beta_l rn_x) and pair_ae[s] the query row's
  // (-s_q s_l / (2 beta_l)), so the accumulator is s_q s_l (dot - rn_x / 2)
  const void* xrn16;
  const float* pair_ae;
  // few-query scan with pair_cnt set: compact outputs at this slot stride
  int out_stride;
  // flat tensor-core scan writing distances instead of a top-k: row q of the
  // (nq, dmat_ld) matrix gets the distance to every database row (IP: the
  // negated inner product, the top-k's key order), dmat_ld a multiple of 128
  float* dmat;
  int64_t dmat_ld;
  // range search
  float radius;
  int64_t* counts;        // count pass: (nq*P)
  const int64_t* offsets; // fill pass: exclusive scan of counts (nq*P)
};

// Tensor-core engine (mf_tc.cu) for the L2 / inner-product top-k scans: items
// of tc_group() queries; a.xq / a.xb are the fp32 (hi) operands, a_lo / b_lo
// their tf32 residuals, a_rows / b_rows their row counts.
bool tc_eligible(int metric, int d, int k, int64_t xb_rows);
// One warp per IVF item of at most few_max_queries() queries (mf_few.cu):
// items from a.items / a.item_total cut into groups of a.group, L2 or inner
// product, d <= 256, k <= 32.
bool few_eligible(int metric, int d, int k);
int few_max_queries();
int launch_few_scan(const ScanArgs& a, int metric, int64_t max_items, int device,
                    cudaStream_t stream);

// True when the tensor-core scan keeps the query tile in tensor memory
// (d <= 128): it then reads raw fp32 queries (a.xq, rows of a.d floats; for
// IVF through a.pairs) and needs neither a_lo nor gathered query rows.
bool tc_raw_queries(int d, int k);
int tc_group();
int launch_tc_scan(const ScanArgs& a, int metric, const float* a_lo, int64_t a_rows,
                   const float* b_lo, int64_t b_rows, int64_t total_items, int device,
                   cudaStream_t stream);
// The fp16 filter scan: IVF items of tc_group() queries, L2, a.k partial slots
// per pair (the smallest upper-bound distances of the list, with row
// positions as labels; a.k <= filter_slots()), A = fp16(scaled query -
// centroid) in tensor memory, B = a.xb as fp16 rows (b_rows of them),
// a.xnorms the rows' squared residual norms.
bool tc_filter_eligible(int d);
int filter_slots();
int launch_tc_filter(const ScanArgs& a, int64_t b_rows, int64_t total_items, int device,
                     cudaStream_t stream);
int launch_tf32_residual(const float* x, int64_t n, int d, float* lo, cudaStream_t stream);
int launch_gather_queries(const float* xq, int d, const int* pairs, const int* n_pairs,
                          int64_t max_pairs, int P, float* g_hi, float* g_lo, cudaStream_t stream);
void set_scan_engine(int engine);
void set_filter_groups(int groups);
int scan_engine();
int read_device_error(int* code);

// Launches the kernel for (metric, kcap, epilogue) on a persistent grid that
// covers `total_items` work items (an upper bound for IVF).
int launch_scan(const ScanArgs& a, int metric, int epilogue, int64_t total_items, int device,
                cudaStream_t stream);

// Smallest supported list capacity >= k, or 0 when k is too large.
int scan_kcap(int k);
constexpr int kMaxK = 256;

// Per-row squared norms.
int launch_norms(const float* x, int64_t n, int d, float* norms, cudaStream_t stream);

// labels[i] = ids[labels[i]] for labels[i] >= 0.
int launch_map_ids(const int64_t* ids, int64_t* labels, int64_t n, cudaStream_t stream);

// Partial top-k merge (nq, parts, k_in) -> (nq, k).
int launch_merge(const float* pd, const int64_t* pl, int64_t nq, int parts, int k_in, int k,
                 float* d, int64_t* l, cudaStream_t stream);
// The same merge over any layout: slot j of part p of query q at
// q * qs + p * ps + j (element strides, one pair per array).
int launch_merge_strided(const float* pd, int64_t d_qs, int64_t d_ps, const int64_t* pl,
                         int64_t l_qs, int64_t l_ps, int64_t nq, int parts, int k_in, int k,
                         float* d, int64_t* l, cudaStream_t stream);

// Flat search plan: splits and workspace.
struct FlatPlan {
  int nqt;
  int splits;
  int64_t rows_per_split;
  size_t bytes;      // workspace for either path (what the size queries report)
  size_t bytes_min;  // without the distance matrix (the fused top-k only)
  int64_t dmat_ld;   // > 0: the distance-matrix path is planned (row stride)
  // tensor cores: the (query tile x 128-row tile) space is cut into `chunks`
  // equal runs of chunk_tiles tiles, one per CTA (0 = items of whole splits)
  int64_t chunk_tiles = 0;
  int64_t tiles_per_qt = 0;
  int chunks = 0;
};
// tq = queries per item (32 for the SIMT scan, tc_group() for tensor cores);
// bytes covers both engines.
// dmat: plan the distance-matrix path where it applies (flat_dmat_ld).
FlatPlan plan_flat(int64_t nq, int64_t nb, int d, int k, int device, int tq = 32,
                   bool dmat = true);
// Row stride of the flat search's distance-matrix path (the tensor-core scan
// writes every query's distances, then one warp per query selects its top-k),
// or 0 where the fused top-k is used: k in [8, 32], 2 to 64 query tiles, and
// a matrix of at most 2 GB. With few query tiles per SM the fused scan cuts
// every tile into pieces whose top-k lists each start empty, and those
// merges (the coarse quantizer of a sharded index: k = nprobe over thousands
// of centroids for a rank's share of the queries) cost more than writing and
// reading the matrix.
int64_t flat_dmat_ld(int64_t nq, int64_t nb, int k);
int launch_dmat_select(const float* dmat, int64_t ld, int64_t nq, int64_t nb, int k,
                       const int64_t* ids, float* D, int64_t* I, cudaStream_t stream);

// Runs flat top-k into (nq, k) outputs using the given workspace. With xb_lo
// (the tf32 residual of xb) the tensor-core engine runs where eligible.
// bound (nq floats, optional): an upper bound on each query's k-th distance;
// rows farther than it are not kept (results may then hold fewer than k).
int run_flat_topk(int device, cudaStream_t stream, const float* xq, int64_t nq, const float* xb,
                  const float* xb_norms, const float* xb_lo, int64_t nb, int d, int metric, int k,
                  const int64_t* ids, float* D, int64_t* I, void* ws, size_t ws_bytes,
                  const float* bound = nullptr);

// IVF list grouping: probes (nq, P) -> pairs grouped by list and items.
struct IvfGroups {
  int* counts;        // nlist
  int* cursors;       // nlist
  int* pair_offsets;  // nlist+1
  int* pairs;         // nq*P
  int2* items;        // nq*P (upper bound)
  int* item_total;    // 1
  int2* items2;       // groups of few queries, when split off (nq*P upper bound)
  int* item_total2;   // 1
  int* counter;       // 1
  int3* plan_sums;    // ceil(nlist / 1024): the multi-block plan's block totals
};
size_t ivf_groups_bytes(int64_t nq, int nlist, int P);
IvfGroups carve_ivf_groups(Carver& c, int64_t nq, int nlist, int P);
int run_ivf_groups(const IvfGroups& g, const int64_t* probes, int64_t nq, int P, int nlist,
                   const int64_t* list_offsets, const int32_t* list_order, int group,
                   cudaStream_t stream);

// bound[q] = pd[(q*P + 0)*k + k-1] (the k-th distance of slot 0).
int launch_extract_bound(const float* pd, int64_t nq, int P, int k, float* bound,
                         cudaStream_t stream);
// Same for a bound computed by the SIMT engine and used by the tensor-core
// engine (L2): adds a margin for their rounding difference, from the query
// norm and the largest norm among the first max_rows rows of probe 0's list.
int launch_extract_bound_slack(const float* pd, int64_t nq, int P, int k, const int64_t* probes,
                               const int64_t* list_offsets, const float* list_norms,
                               const float* qnorms, int64_t max_rows, int d, float* bound,
                               cudaStream_t stream);

// Exclusive scan of n int64 counts into out (n+1 entries; out[n] = total).
int launch_exclusive_scan_i64(const int64_t* in, int64_t n, int64_t* out, cudaStream_t stream);

// Accumulation probes of the fp16 tensor-core products (diagnostics):
// tcgen05 (A 128 x d in tensor memory, B 128 x d by TMA; out 128 x 128) and
// mma.sync m16n8k16 (A 16 x d, B 8 x d; out 16 x 8), fp32 accumulation.
int launch_f16_probe_tc(const void* a, const void* b, int d, float* out, cudaStream_t stream);
int launch_f16_probe_mma(const void* a, const void* b, int d, float* out, cudaStream_t stream);

}  // namespace mf
