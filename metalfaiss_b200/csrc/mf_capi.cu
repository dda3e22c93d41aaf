// extern "C" entry points (include/metalfaiss_b200.h): argument checks,
// workspace planning and kernel sequencing. No entry point allocates memory.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "mf_filter.cuh"
#include "mf_ivf.cuh"
#include "mf_scan.cuh"

namespace mf {

namespace {
thread_local std::string g_last_error;
std::mutex g_sm_mu;
int g_sms[64] = {0};
}  // namespace

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MF_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e),
              cudaGetErrorString(e));
}

void clear_error() { g_last_error.clear(); }

DeviceGuard::DeviceGuard(int device) {
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    status = fail(MF_ERR_INVALID_ARGS, "invalid CUDA device %d (%d visible)", device, n);
    return;
  }
  if (prev != device) {
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) status = cuda_fail(e, "cudaSetDevice");
  }
}

DeviceGuard::~DeviceGuard() {
  int cur = -1;
  if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
}

int check_device_ptr(const void* p, const char* name, bool allow_null) {
  if (p == nullptr) {
    if (allow_null) return MF_OK;
    return fail(MF_ERR_INVALID_ARGS, "%s is NULL", name);
  }
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MF_ERR_INVALID_ARGS, "%s is not a CUDA pointer (%s)", name, cudaGetErrorName(e));
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return fail(MF_ERR_INVALID_ARGS, "%s must be device memory (got memory type %d)", name,
                (int)attr.type);
  int cur = -1;
  cudaGetDevice(&cur);
  if (attr.type == cudaMemoryTypeDevice && attr.device != cur)
    return fail(MF_ERR_INVALID_ARGS, "%s lives on device %d, call targets device %d", name,
                attr.device, cur);
  if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0)
    return fail(MF_ERR_INVALID_ARGS, "%s is not 16-byte aligned", name);
  return MF_OK;
}

int num_sms(int device) {
  if (device < 0 || device >= 64) return 148;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  if (g_sms[device] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || v <= 0)
      v = 148;
    g_sms[device] = v;
  }
  return g_sms[device];
}

namespace {

int check_common(int d, int metric, int k, bool need_k) {
  MF_CHECK(d > 0 && d % 4 == 0, MF_ERR_INVALID_ARGS,
           "d=%d must be a positive multiple of 4 (pad rows with zeros)", d);
  MF_CHECK(metric >= 0 && metric <= 3, MF_ERR_METRIC,
           "metric %d is not one of INNER_PRODUCT(0), L2(1), L1(2), LINF(3)", metric);
  if (need_k)
    MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d outside [1, %d]", k, kMaxK);
  return MF_OK;
}

// ---- IVF workspace layout shared by search / range passes
struct IvfWs {
  float* qn;
  float* coarse_d;
  int64_t* coarse_l;
  void* flat_ws;
  size_t flat_bytes;
  IvfGroups g;
  float* pd;
  int64_t* pl;
  int64_t* pair_counts;
  int64_t* pair_offsets64;
  float* bound;      // per-query bound from the first rows of the nearest list
  float* g_hi;       // gathered query rows per (query, probe) pair (tensor cores)
  float* g_lo;
  float* cent_lo;    // tf32 residuals of the centroids (coarse step, tensor cores)
  FilterPairs fp;    // filter search: per (query, probe) pair
};

// mode: 0 = top-k search, 1 = preassigned top-k, 2 = range, 3 = filter search,
// 4 = preassigned filter search
IvfWs carve_ivf(Carver& c, int64_t nq, int nlist, int P, int d, int k, int mode, int device) {
  IvfWs w{};
  w.qn = c.take<float>(nq);
  if (mode != 1 && mode != 4) {
    w.coarse_d = c.take<float>((size_t)nq * P);
    w.coarse_l = c.take<int64_t>((size_t)nq * P);
    FlatPlan fp = plan_flat(nq, nlist, d, P, device);
    w.flat_bytes = fp.bytes;
    w.flat_ws = c.take<char>(fp.bytes);
    w.cent_lo = c.take<float>((size_t)nlist * d);
  }
  w.g = carve_ivf_groups(c, nq, nlist, P);
  if (mode == 2) {
    w.pair_counts = c.take<int64_t>((size_t)nq * P);
    w.pair_offsets64 = c.take<int64_t>((size_t)nq * P + 1);
  } else if (mode >= 3) {
    // the filter pass keeps filter_slots() slots per pair (>= k)
    w.pd = c.take<float>((size_t)nq * P * filter_slots());
    w.pl = c.take<int64_t>((size_t)nq * P * filter_slots());
    w.bound = c.take<float>((size_t)nq);
    w.fp.qn = c.take<float>((size_t)nq * P);
    w.fp.thr = c.take<float>((size_t)nq * P);
    w.fp.e = c.take<float>((size_t)nq * P);
    w.fp.sq = c.take<float>((size_t)nq * P);
    w.fp.sc = c.take<float>((size_t)nq * P);
    w.fp.ae = c.take<float>((size_t)nq * P);
    w.fp.cnt = c.take<int>((size_t)nq * P);
  } else {
    w.pd = c.take<float>((size_t)nq * P * k);
    w.pl = c.take<int64_t>((size_t)nq * P * k);
    w.bound = c.take<float>((size_t)nq);
    w.g_hi = c.take<float>((size_t)nq * P * d);
    w.g_lo = c.take<float>((size_t)nq * P * d);
  }
  return w;
}

int effective_nprobe(int nprobe, int nlist) { return nprobe < nlist ? nprobe : nlist; }

int coarse_metric(int metric) {
  return metric == MF_METRIC_INNER_PRODUCT ? MF_METRIC_INNER_PRODUCT : MF_METRIC_L2;
}

// bound_out != NULL: run only the bound pass and write each query's bound
// there (+inf where its first probe holds no rows). bound_in != NULL: skip the
// bound pass and filter the all-probes pass by bound_in (a bound computed
// elsewhere, e.g. the minimum over the ranks that hold the lists).
// The items split off as few-query groups (w.g.items2): one warp per item
// where the shape allows, else the SIMT scan.
int scan_small_items(const ScanArgs& base, const IvfWs& w, int metric, int64_t max_items,
                     int device, cudaStream_t stream, int group) {
  ScanArgs sa = base;
  sa.items = w.g.items2;
  sa.item_total = w.g.item_total2;
  sa.group = group;
  if (few_eligible(metric, sa.d, sa.k)) return launch_few_scan(sa, metric, max_items, device, stream);
  return launch_scan(sa, metric, kEpiTopK, max_items, device, stream);
}

// Rows of a query's nearest list that the bound pass scans (at most).
constexpr int64_t kBoundRows = 128;

int ivf_scan_topk(int device, cudaStream_t stream, const IvfWs& w, const float* xq, int64_t nq,
                  const int64_t* probes, int P, int nlist, const int64_t* list_offsets,
                  const float* list_vecs, const float* list_norms, const float* list_lo,
                  const int64_t* list_ids, int64_t ntotal, const int32_t* list_order, int d,
                  int metric, int k, float* D, int64_t* I, float* bound_out = nullptr,
                  const float* bound_in = nullptr) {
  // tensor cores: where the shape allows, given the rows' tf32 residuals or,
  // for d <= 128, deriving them in the kernel
  const bool tc = tc_eligible(metric, d, k, ntotal) && (list_lo != nullptr || tc_raw_queries(d, k));
  if (metric == MF_METRIC_L2) MF_TRY(launch_norms(xq, nq, d, w.qn, stream));
  ScanArgs a{};
  a.xq = xq;
  a.qnorms = w.qn;
  a.xb = list_vecs;
  a.xnorms = list_norms;
  a.ids = list_ids;
  a.d = d;
  a.k = k;
  a.nq = nq;
  a.P = P;
  a.flat = 0;
  a.items = w.g.items;
  a.item_total = w.g.item_total;
  a.list_offsets = list_offsets;
  a.pair_offsets = w.g.pair_offsets;
  a.pairs = w.g.pairs;
  a.counter = w.g.counter;
  a.out_d = w.pd;
  a.out_l = w.pl;
  a.direct = 0;
  // Two phases. Phase 1 scans only the first kBoundRows rows of every query's
  // nearest list (probe 0); the k-th distance found there is an upper bound
  // on the query's final k-th distance. Phase 2 scans all probes, keeping
  // only candidates within the bound, so most rows of the farther lists never
  // enter the top-k merges. For L2 phase 1 runs on the SIMT engine (its
  // one-tile items are cheaper there); the bound then carries a margin for
  // the engines' rounding difference, so phase 2 still drops no row that
  // belongs to the top-k.
  constexpr int kSmallGroup = 16;
  // bound pass groups: the SIMT scan's 32 queries per item
  const int few_group = kScanTQ;
  const int phases = (bound_out || bound_in) ? 1 : (P > 1 ? 2 : 1);
  float* const bound_dst = bound_out ? bound_out : w.bound;
  for (int ph = 0; ph < phases; ++ph) {
    const bool bounding = bound_out != nullptr || (phases == 2 && ph == 0);
    const bool simt_bound = bounding && tc && metric == MF_METRIC_L2;
    const bool use_tc = tc && !simt_bound;
    // Tensor-core pass: groups of up to 128 queries per list, except that a
    // list probed by at most kSmallGroup queries goes to the few-query scan:
    // a 128-query tile would be mostly padding, and those rows' bytes, not
    // their arithmetic, bound the work.
    // (L2 only: the bound then carries the margin that covers both engines).
    // The SIMT bound pass splits off its small groups the same way.
    const bool few_ok = few_eligible(metric, d, k) && metric == MF_METRIC_L2;
    const int small_max = (use_tc && !bounding && metric == MF_METRIC_L2) ? kSmallGroup
                          : (simt_bound && few_ok) ? few_max_queries() : 0;
    const int grp = use_tc ? tc_group() : (small_max > 0 ? few_group : kScanTQ);
    MF_TRY(run_ivf_groups_ex(w.g, probes, nq, P, nlist, list_offsets, list_order, w.pd, w.pl, k,
                             nullptr, grp, stream, 0, bounding ? 1 : P, small_max));
    a.max_rows = bounding ? kBoundRows : 0;
    a.bound = bound_in ? bound_in : ((phases == 2 && ph == 1) ? w.bound : nullptr);
    if (use_tc && tc_raw_queries(d, k)) {
      // the scan loads each item's queries itself (through a.pairs)
      MF_TRY(launch_tc_scan(a, metric, nullptr, nq, list_lo, ntotal, nq * P, device, stream));
      if (small_max > 0)
        MF_TRY(scan_small_items(a, w, metric, nq * P, device, stream, tc_group()));
    } else if (use_tc) {
      // A operand: the queries of every (query, probe) pair, gathered in list order
      MF_TRY(launch_gather_queries(xq, d, w.g.pairs, w.g.pair_offsets + nlist, nq * P, P, w.g_hi,
                                   w.g_lo, stream));
      a.xq = w.g_hi;
      MF_TRY(launch_tc_scan(a, metric, w.g_lo, nq * P, list_lo, ntotal, nq * P, device, stream));
      a.xq = xq;
      if (small_max > 0)
        MF_TRY(scan_small_items(a, w, metric, nq * P, device, stream, tc_group()));
    } else if (small_max > 0) {
      // bound pass: a list that is the nearest for at most few_max_queries()
      // queries goes to the few-query scan, the others, in groups of
      // few_group queries, to the SIMT scan
      ScanArgs ga = a;
      ga.group = few_group;
      MF_TRY(launch_scan(ga, metric, kEpiTopK, nq * P, device, stream));
      MF_TRY(scan_small_items(ga, w, metric, nq * P, device, stream, few_group));
    } else {
      MF_TRY(launch_scan(a, metric, kEpiTopK, nq * P, device, stream));
    }
    if (simt_bound)
      MF_TRY(launch_extract_bound_slack(w.pd, nq, P, k, probes, list_offsets, list_norms, w.qn,
                                        kBoundRows, d, bound_dst, stream));
    else if (bounding)
      MF_TRY(launch_extract_bound(w.pd, nq, P, k, bound_dst, stream));
  }
  if (bound_out) return MF_OK;
  MF_TRY(launch_merge(w.pd, w.pl, nq, P, k, k, D, I, stream));
  return MF_OK;
}

// The filter search (L2): the bound pass (unless bound_in is given), the
// per-pair scales and error bounds, the fp16 filter pass over every probed list in
// groups of up to 128 queries, and the exact refinement into (D, I). The
// bound pass runs on the SIMT engines with the margin that also covers the
// refinement's rounding (filter_eligible requires the tensor-core shape for it).
// Lists probed by at most this many queries go to the few-query pass in the
// filter search (0: every list to the tensor-core pass).
int g_filter_small_group = 16;

int ivf_filter_topk(int device, cudaStream_t stream, const IvfWs& w, const float* xq, int64_t nq,
                    const int64_t* probes, int P, int nlist, const int64_t* list_offsets,
                    const float* list_vecs, const float* list_norms, const float* list_lo,
                    const int64_t* list_ids, int64_t ntotal, const int32_t* list_order,
                    const void* list_f16, const float* list_rnorms, const void* list_rn16,
                    const float* list_stats, const float* centroids, int d, int k, float* D,
                    int64_t* I, const float* bound_in) {
  const int S = filter_slots_for(k);
  if (bound_in) {
    MF_TRY(launch_norms(xq, nq, d, w.qn, stream));
  } else {
    MF_TRY(ivf_scan_topk(device, stream, w, xq, nq, probes, P, nlist, list_offsets, list_vecs,
                         list_norms, list_lo, list_ids, ntotal, list_order, d, MF_METRIC_L2, k,
                         nullptr, nullptr, w.bound));
  }
  const float* bound = bound_in ? bound_in : w.bound;
  MF_TRY(launch_filter_pairs(xq, w.qn, nq, P, d, probes, list_offsets, nlist, centroids,
                             list_stats, bound, w.fp, stream));
  // (pairs that are not scanned have no kept slots: launch_filter_pairs).
  // A list probed by at most kSmallGroup queries goes to the few-query scan
  // instead (a 128-query tile would be mostly padding; those rows' bytes
  // bound the work), in its filter form: the same fp16 rows, upper bounds and
  // slots.
  const int small_max = few_eligible(MF_METRIC_L2, d, k) ? g_filter_small_group : 0;
  MF_TRY(run_ivf_groups_ex(w.g, probes, nq, P, nlist, list_offsets, list_order, nullptr, nullptr,
                           0, nullptr, tc_group(), stream, 0, P, small_max));
  ScanArgs a{};
  a.xq = xq;
  a.qnorms = w.qn;
  a.xb = reinterpret_cast<const float*>(list_f16);  // fp16 rows, read only by TMA
  a.xnorms = list_rnorms;
  a.ids = nullptr;  // slots carry row positions for the refinement
  a.d = d;
  a.k = S;
  a.nq = nq;
  a.P = P;
  a.flat = 0;
  a.items = w.g.items;
  a.item_total = w.g.item_total;
  a.list_offsets = list_offsets;
  a.pair_offsets = w.g.pair_offsets;
  a.pairs = w.g.pairs;
  a.counter = w.g.counter;
  a.out_d = w.pd;
  a.out_l = w.pl;
  a.pair_qn = w.fp.qn;
  a.pair_thr = w.fp.thr;
  a.pair_sq = w.fp.sq;
  a.pair_sc = w.fp.sc;
  a.pair_cnt = w.fp.cnt;
  a.centroids = centroids;
  a.xrn16 = list_rn16;
  a.pair_ae = w.fp.ae;
  MF_TRY(launch_tc_filter(a, ntotal, nq * P, device, stream));
  if (small_max > 0) {
    ScanArgs fa{};
    fa.xq = xq;
    fa.qnorms = w.qn;
    fa.xb = reinterpret_cast<const float*>(list_f16);
    fa.xnorms = list_rnorms;
    fa.ids = nullptr;
    fa.d = d;
    fa.k = S;
    fa.nq = nq;
    fa.P = P;
    fa.flat = 0;
    fa.items = w.g.items2;
    fa.item_total = w.g.item_total2;
    fa.group = tc_group();
    fa.list_offsets = list_offsets;
    fa.pair_offsets = w.g.pair_offsets;
    fa.pairs = w.g.pairs;
    fa.counter = w.g.counter;
    fa.out_d = w.pd;
    fa.out_l = w.pl;
    fa.pair_qn = w.fp.qn;
    fa.pair_thr = w.fp.thr;
    fa.pair_sq = w.fp.sq;
    fa.pair_sc = w.fp.sc;
    fa.pair_cnt = w.fp.cnt;
    fa.centroids = centroids;
    fa.out_stride = S;
    MF_TRY(launch_few_scan(fa, MF_METRIC_L2, nq * P, device, stream));
  }
  RefineArgs f{};
  f.xq = xq;
  f.qnorms = w.qn;
  f.nq = nq;
  f.d = d;
  f.P = P;
  f.k = k;
  f.slots = S;
  f.pd = w.pd;
  f.pl = w.pl;
  f.cnt = w.fp.cnt;
  f.pair_e = w.fp.e;
  f.bound = bound;
  f.probes = probes;
  f.offsets = list_offsets;
  f.xb = list_vecs;
  f.xnorms = list_norms;
  f.ids = list_ids;
  f.D = D;
  f.I = I;
  return launch_filter_refine(f, stream);
}

bool filter_eligible(int d, int k, int64_t ntotal) {
  return tc_filter_eligible(d) && k >= 1 && 2 * k <= filter_slots() &&
         tc_eligible(MF_METRIC_L2, d, k, ntotal) && tc_raw_queries(d, k);
}

int check_filter_bank(const void* list_f16, const float* list_rnorms, const void* list_rn16,
                      const float* list_stats, const float* centroids) {
  MF_TRY(check_device_ptr(list_f16, "list_f16"));
  MF_TRY(check_device_ptr(list_rnorms, "list_rnorms"));
  MF_TRY(check_device_ptr(list_rn16, "list_rn16"));
  MF_TRY(check_device_ptr(list_stats, "list_stats"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  return MF_OK;
}

int check_ivf_lists(const int64_t* list_offsets, const float* list_vecs, const float* list_norms,
                    const int64_t* list_ids, const int32_t* list_order, int metric) {
  MF_TRY(check_device_ptr(list_offsets, "list_offsets"));
  MF_TRY(check_device_ptr(list_vecs, "list_vecs", true));
  MF_TRY(check_device_ptr(list_ids, "list_ids", true));
  MF_TRY(check_device_ptr(list_norms, "list_norms", metric != MF_METRIC_L2));
  MF_TRY(check_device_ptr(list_order, "list_order", true));
  return MF_OK;
}

}  // namespace
}  // namespace mf

using namespace mf;

#define MF_ENTER(device)                     \
  clear_error();                             \
  DeviceGuard _guard(device);                \
  if (_guard.status != MF_OK) return _guard.status

extern "C" {

int mf_version(void) { return 100; }

const char* mf_last_error(void) { return g_last_error.c_str(); }

int mf_max_k(void) { return kMaxK; }

int mf_ivf_bound_rows(void) { return (int)kBoundRows; }

int mf_diag_f16_dot(int device, void* stream, int engine, const void* a, const void* b, int d,
                    float* out) {
  MF_ENTER(device);
  MF_CHECK(engine == 0 || engine == 1, MF_ERR_INVALID_ARGS,
           "engine %d: 0 = tcgen05, 1 = mma.sync", engine);
  MF_TRY(check_device_ptr(a, "a"));
  MF_TRY(check_device_ptr(b, "b"));
  MF_TRY(check_device_ptr(out, "out"));
  return engine == 0 ? launch_f16_probe_tc(a, b, d, out, (cudaStream_t)stream)
                     : launch_f16_probe_mma(a, b, d, out, (cudaStream_t)stream);
}

int mf_flat_engine(int metric, int d, int k, int64_t nb, int has_residuals) {
  clear_error();
  return (tc_eligible(metric, d, k, nb) && (has_residuals != 0 || tc_raw_queries(d, k))) ? 1
                                                                                          : 0;
}

int mf_vector_norms(int device, void* stream, const float* x, int64_t n, int d, float* norms) {
  MF_ENTER(device);
  MF_CHECK(n >= 0 && d > 0 && d % 4 == 0, MF_ERR_INVALID_ARGS, "bad shape n=%lld d=%d",
           (long long)n, d);
  if (n == 0) return MF_OK;
  MF_TRY(check_device_ptr(x, "x"));
  MF_TRY(check_device_ptr(norms, "norms"));
  return launch_norms(x, n, d, norms, (cudaStream_t)stream);
}

int mf_flat_search_workspace_size(int64_t nq, int64_t nb, int d, int metric, int k,
                                  size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_common(d, metric, k, true));
  int dev = 0;
  cudaGetDevice(&dev);
  *bytes = plan_flat(nq, nb, d, k, dev).bytes;
  return MF_OK;
}

int mf_flat_search(int device, void* stream, const float* xq, int64_t nq, const float* xb,
                   const float* xb_norms, const float* xb_lo, int64_t nb, int d, int metric, int k,
                   const int64_t* ids, float* distances, int64_t* labels, void* workspace,
                   size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nq >= 0 && nb >= 0, MF_ERR_INVALID_ARGS, "negative sizes");
  MF_CHECK(nb < (1ll << 31) - 1, MF_ERR_INVALID_ARGS, "nb=%lld exceeds 2^31-2 rows per call",
           (long long)nb);
  MF_CHECK(nq < (1ll << 31) / 2, MF_ERR_INVALID_ARGS, "nq too large");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  MF_TRY(check_device_ptr(ids, "ids", true));
  if (metric == MF_METRIC_L2) MF_TRY(check_device_ptr(xb_norms, "xb_norms", nb == 0));
  MF_TRY(check_device_ptr(workspace, "workspace", true));
  MF_TRY(check_device_ptr(xb_lo, "xb_lo", true));
  return run_flat_topk(device, (cudaStream_t)stream, xq, nq, xb, xb_norms, xb_lo, nb, d, metric,
                       k, ids, distances, labels, workspace, workspace_bytes);
}

int mf_flat_search_bounded(int device, void* stream, const float* xq, int64_t nq,
                           const float* xb, const float* xb_norms, const float* xb_lo, int64_t nb,
                           int d, int metric, int k, const int64_t* ids, const float* bound,
                           float* distances, int64_t* labels, void* workspace,
                           size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nq >= 0 && nb >= 0, MF_ERR_INVALID_ARGS, "negative sizes");
  MF_CHECK(nb < (1ll << 31) - 1, MF_ERR_INVALID_ARGS, "nb=%lld exceeds 2^31-2 rows per call",
           (long long)nb);
  MF_CHECK(nq < (1ll << 31) / 2, MF_ERR_INVALID_ARGS, "nq too large");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(bound, "bound"));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  MF_TRY(check_device_ptr(ids, "ids", true));
  if (metric == MF_METRIC_L2) MF_TRY(check_device_ptr(xb_norms, "xb_norms", nb == 0));
  MF_TRY(check_device_ptr(workspace, "workspace", true));
  MF_TRY(check_device_ptr(xb_lo, "xb_lo", true));
  return run_flat_topk(device, (cudaStream_t)stream, xq, nq, xb, xb_norms, xb_lo, nb, d, metric,
                       k, ids, distances, labels, workspace, workspace_bytes, bound);
}

int mf_ivf_search_workspace_size(int64_t nq, int nlist, int nprobe, int d, int metric, int k,
                                 size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  int dev = 0;
  cudaGetDevice(&dev);
  Carver c(nullptr, 0);
  carve_ivf(c, nq, nlist, effective_nprobe(nprobe, nlist), d, k, 0, dev);
  *bytes = c.used;
  return MF_OK;
}

int mf_ivf_search(int device, void* stream, const float* xq, int64_t nq,
                  const float* centroids, const float* centroid_norms, int nlist, int nprobe,
                  const int64_t* list_offsets, const float* list_vecs, const float* list_norms,
                  const float* list_lo, const int64_t* list_ids, int64_t ntotal,
                  const int32_t* list_order, int d, int metric, int k, float* distances,
                  int64_t* labels, void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nlist >= 1, MF_ERR_INVALID_ARGS, "nlist=%d", nlist);
  MF_CHECK(nprobe >= 1, MF_ERR_INVALID_ARGS, "nprobe must be positive (got %d)", nprobe);
  const int P = effective_nprobe(nprobe, nlist);
  MF_CHECK(P <= kMaxK, MF_ERR_INVALID_ARGS, "nprobe=%d exceeds %d", P, kMaxK);
  MF_CHECK(nq >= 0 && nq * P < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  MF_TRY(check_device_ptr(centroid_norms, "centroid_norms", coarse_metric(metric) != MF_METRIC_L2));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, list_ids, list_order, metric));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, P, d, k, 0, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "IVF search workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  cudaStream_t s = (cudaStream_t)stream;
  const float* cent_lo = nullptr;
  // the centroids' residuals (8 MB at 16384 x 128): loading them beats deriving them
  if (tc_eligible(coarse_metric(metric), d, P, nlist)) {
    MF_TRY(launch_tf32_residual(centroids, nlist, d, w.cent_lo, s));
    cent_lo = w.cent_lo;
  }
  MF_TRY(run_flat_topk(device, s, xq, nq, centroids, centroid_norms, cent_lo, nlist, d,
                       coarse_metric(metric), P, nullptr, w.coarse_d, w.coarse_l, w.flat_ws,
                       w.flat_bytes));
  return ivf_scan_topk(device, s, w, xq, nq, w.coarse_l, P, nlist, list_offsets, list_vecs,
                       list_norms, list_lo, list_ids, ntotal, list_order, d, metric, k, distances,
                       labels);
}

int mf_ivf_search_preassigned_workspace_size(int64_t nq, int nlist, int nprobe, int d,
                                             int metric, int k, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  int dev = 0;
  cudaGetDevice(&dev);
  Carver c(nullptr, 0);
  carve_ivf(c, nq, nlist, nprobe, d, k, 1, dev);
  *bytes = c.used;
  return MF_OK;
}

int mf_ivf_search_preassigned(int device, void* stream, const float* xq, int64_t nq,
                              const int64_t* probes, int nprobe, int nlist,
                              const int64_t* list_offsets, const float* list_vecs,
                              const float* list_norms, const float* list_lo,
                              const int64_t* list_ids, int64_t ntotal, const int32_t* list_order,
                              int d, int metric, int k, float* distances, int64_t* labels,
                              void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  MF_CHECK(nq >= 0 && nq * nprobe < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(probes, "probes"));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, list_ids, list_order, metric));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, nprobe, d, k, 1, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  return ivf_scan_topk(device, (cudaStream_t)stream, w, xq, nq, probes, nprobe, nlist,
                       list_offsets, list_vecs, list_norms, list_lo, list_ids, ntotal, list_order,
                       d, metric, k, distances, labels);
}

namespace {
int ivf_preassigned_entry(int device, void* stream, const float* xq, int64_t nq,
                          const int64_t* probes, int nprobe, int nlist, const int64_t* list_offsets,
                          const float* list_vecs, const float* list_norms, const float* list_lo,
                          const int64_t* list_ids, int64_t ntotal, const int32_t* list_order, int d,
                          int metric, int k, float* distances, int64_t* labels, float* bound_out,
                          const float* bound_in, void* workspace, size_t workspace_bytes) {
  MF_TRY(check_common(d, metric, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  MF_CHECK(nq >= 0 && nq * nprobe < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(probes, "probes"));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, list_ids, list_order, metric));
  if (bound_out) {
    MF_TRY(check_device_ptr(bound_out, "bound"));
  } else {
    MF_TRY(check_device_ptr(distances, "distances"));
    MF_TRY(check_device_ptr(labels, "labels"));
  }
  if (bound_in) MF_TRY(check_device_ptr(bound_in, "bound"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, nprobe, d, k, 1, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  return ivf_scan_topk(device, (cudaStream_t)stream, w, xq, nq, probes, nprobe, nlist,
                       list_offsets, list_vecs, list_norms, list_lo, list_ids, ntotal, list_order,
                       d, metric, k, distances, labels, bound_out, bound_in);
}
}  // namespace

int mf_ivf_probe_bound(int device, void* stream, const float* xq, int64_t nq,
                       const int64_t* probes, int nprobe, int nlist, const int64_t* list_offsets,
                       const float* list_vecs, const float* list_norms, const float* list_lo,
                       const int64_t* list_ids, int64_t ntotal, const int32_t* list_order, int d,
                       int metric, int k, float* bound, void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  return ivf_preassigned_entry(device, stream, xq, nq, probes, nprobe, nlist, list_offsets,
                               list_vecs, list_norms, list_lo, list_ids, ntotal, list_order, d,
                               metric, k, nullptr, nullptr, bound, nullptr, workspace,
                               workspace_bytes);
}

int mf_ivf_search_bounded(int device, void* stream, const float* xq, int64_t nq,
                          const int64_t* probes, int nprobe, int nlist,
                          const int64_t* list_offsets, const float* list_vecs,
                          const float* list_norms, const float* list_lo, const int64_t* list_ids,
                          int64_t ntotal, const int32_t* list_order, int d, int metric, int k,
                          const float* bound, float* distances, int64_t* labels, void* workspace,
                          size_t workspace_bytes) {
  MF_ENTER(device);
  return ivf_preassigned_entry(device, stream, xq, nq, probes, nprobe, nlist, list_offsets,
                               list_vecs, list_norms, list_lo, list_ids, ntotal, list_order, d,
                               metric, k, distances, labels, nullptr, bound, workspace,
                               workspace_bytes);
}

int mf_ivf_filter_eligible(int d, int k, int64_t ntotal) {
  clear_error();
  return filter_eligible(d, k, ntotal) ? 1 : 0;
}

int mf_ivf_filter_bank(int device, void* stream, int nlist, int d, const int64_t* list_offsets,
                       const float* list_vecs, const float* list_norms, const float* centroids,
                       int64_t ntotal, void* list_f16, float* list_rnorms, void* list_rn16,
                       float* list_stats) {
  MF_ENTER(device);
  // the filter search's shapes only (mf_ivf_filter_eligible): its scan reads
  // 128-byte fp16 tiles (d >= 64) and its refinement one float4 per lane
  // (d <= 128)
  MF_CHECK(nlist >= 1 && d >= 64 && d <= 128 && d % 8 == 0, MF_ERR_INVALID_ARGS,
           "filter bank: nlist=%d, d=%d (the filter search takes 64 <= d <= 128, a multiple "
           "of 8)", nlist, d);
  MF_TRY(check_device_ptr(list_offsets, "list_offsets"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  MF_TRY(check_device_ptr(list_stats, "list_stats"));
  if (ntotal > 0) {
    MF_TRY(check_device_ptr(list_vecs, "list_vecs"));
    MF_TRY(check_device_ptr(list_norms, "list_norms"));
    MF_TRY(check_device_ptr(list_f16, "list_f16"));
    MF_TRY(check_device_ptr(list_rnorms, "list_rnorms"));
    MF_TRY(check_device_ptr(list_rn16, "list_rn16"));
  }
  return launch_filter_bank(nlist, d, list_offsets, list_vecs, list_norms, centroids, list_f16,
                            list_rnorms, list_stats, list_rn16, (cudaStream_t)stream);
}

int mf_ivf_search_filtered_workspace_size(int64_t nq, int nlist, int nprobe, int d, int k,
                                          size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_common(d, MF_METRIC_L2, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  int dev = 0;
  cudaGetDevice(&dev);
  Carver c(nullptr, 0);
  carve_ivf(c, nq, nlist, effective_nprobe(nprobe, nlist), d, k, 3, dev);
  *bytes = c.used;
  return MF_OK;
}

int mf_ivf_search_filtered(int device, void* stream, const float* xq, int64_t nq,
                           const float* centroids, const float* centroid_norms, int nlist,
                           int nprobe, const int64_t* list_offsets, const float* list_vecs,
                           const float* list_norms, const float* list_lo,
                           const int64_t* list_ids, int64_t ntotal, const int32_t* list_order,
                           const void* list_f16, const float* list_rnorms,
                           const void* list_rn16, const float* list_stats, int d, int k,
                           float* distances,
                           int64_t* labels, void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, MF_METRIC_L2, k, true));
  MF_CHECK(nlist >= 1, MF_ERR_INVALID_ARGS, "nlist=%d", nlist);
  MF_CHECK(nprobe >= 1, MF_ERR_INVALID_ARGS, "nprobe must be positive (got %d)", nprobe);
  const int P = effective_nprobe(nprobe, nlist);
  MF_CHECK(P <= kMaxK, MF_ERR_INVALID_ARGS, "nprobe=%d exceeds %d", P, kMaxK);
  MF_CHECK(nq >= 0 && nq * P < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  MF_CHECK(filter_eligible(d, k, ntotal), MF_ERR_INVALID_ARGS,
           "the filter search does not take d=%d, k=%d, ntotal=%lld (mf_ivf_filter_eligible)", d,
           k, (long long)ntotal);
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(centroid_norms, "centroid_norms"));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, list_ids, list_order,
                         MF_METRIC_L2));
  MF_TRY(check_filter_bank(list_f16, list_rnorms, list_rn16, list_stats, centroids));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, P, d, k, 3, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "IVF filter search workspace too small: %zu < %zu bytes",
           workspace_bytes, c.used);
  cudaStream_t s = (cudaStream_t)stream;
  const float* cent_lo = nullptr;
  if (tc_eligible(MF_METRIC_L2, d, P, nlist)) {
    MF_TRY(launch_tf32_residual(centroids, nlist, d, w.cent_lo, s));
    cent_lo = w.cent_lo;
  }
  MF_TRY(run_flat_topk(device, s, xq, nq, centroids, centroid_norms, cent_lo, nlist, d,
                       MF_METRIC_L2, P, nullptr, w.coarse_d, w.coarse_l, w.flat_ws, w.flat_bytes));
  return ivf_filter_topk(device, s, w, xq, nq, w.coarse_l, P, nlist, list_offsets, list_vecs,
                         list_norms, list_lo, list_ids, ntotal, list_order, list_f16, list_rnorms,
                         list_rn16, list_stats, centroids, d, k, distances, labels, nullptr);
}

int mf_ivf_search_bounded_filtered_workspace_size(int64_t nq, int nlist, int nprobe, int d,
                                                  int k, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_TRY(check_common(d, MF_METRIC_L2, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  int dev = 0;
  cudaGetDevice(&dev);
  Carver c(nullptr, 0);
  carve_ivf(c, nq, nlist, nprobe, d, k, 4, dev);
  *bytes = c.used;
  return MF_OK;
}

int mf_ivf_search_bounded_filtered(int device, void* stream, const float* xq, int64_t nq,
                                   const int64_t* probes, int nprobe, int nlist,
                                   const int64_t* list_offsets, const float* list_vecs,
                                   const float* list_norms, const int64_t* list_ids,
                                   int64_t ntotal, const int32_t* list_order, const void* list_f16,
                                   const float* list_rnorms, const void* list_rn16,
                                   const float* list_stats,
                                   const float* centroids, int d, int k, const float* bound,
                                   float* distances, int64_t* labels, void* workspace,
                                   size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, MF_METRIC_L2, k, true));
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  MF_CHECK(nq >= 0 && nq * nprobe < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  MF_CHECK(filter_eligible(d, k, ntotal), MF_ERR_INVALID_ARGS,
           "the filter search does not take d=%d, k=%d, ntotal=%lld (mf_ivf_filter_eligible)", d,
           k, (long long)ntotal);
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(probes, "probes"));
  MF_TRY(check_device_ptr(bound, "bound"));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, list_ids, list_order,
                         MF_METRIC_L2));
  MF_TRY(check_filter_bank(list_f16, list_rnorms, list_rn16, list_stats, centroids));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, nprobe, d, k, 4, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "workspace too small: %zu < %zu bytes", workspace_bytes,
           c.used);
  return ivf_filter_topk(device, (cudaStream_t)stream, w, xq, nq, probes, nprobe, nlist,
                         list_offsets, list_vecs, list_norms, nullptr, list_ids, ntotal,
                         list_order, list_f16, list_rnorms, list_rn16, list_stats, centroids, d, k,
                         distances,
                         labels, bound);
}

int mf_ivf_filter_rescans(int device, int64_t* count, int reset) {
  MF_ENTER(device);
  MF_CHECK(count != nullptr, MF_ERR_INVALID_ARGS, "count is NULL");
  unsigned long long v = 0;
  MF_TRY(read_filter_rescans(&v, reset != 0));
  *count = (int64_t)v;
  return MF_OK;
}

int mf_topk_merge(int device, void* stream, const float* part_distances,
                  const int64_t* part_labels, int64_t nq, int parts, int k_in, int k,
                  float* distances, int64_t* labels) {
  MF_ENTER(device);
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d outside [1, %d]", k, kMaxK);
  MF_CHECK(parts >= 1 && k_in >= 0 && nq >= 0, MF_ERR_INVALID_ARGS, "bad merge shape");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(part_distances, "part_distances", k_in == 0));
  MF_TRY(check_device_ptr(part_labels, "part_labels", k_in == 0));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  return launch_merge(part_distances, part_labels, nq, parts, k_in, k, distances, labels,
                      (cudaStream_t)stream);
}

int mf_topk_merge_strided(int device, void* stream, const float* part_distances,
                          int64_t dist_query_stride, int64_t dist_part_stride,
                          const int64_t* part_labels, int64_t label_query_stride,
                          int64_t label_part_stride, int64_t nq, int parts, int k_in, int k,
                          float* distances, int64_t* labels) {
  MF_ENTER(device);
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d outside [1, %d]", k, kMaxK);
  MF_CHECK(parts >= 1 && k_in >= 0 && nq >= 0, MF_ERR_INVALID_ARGS, "bad merge shape");
  MF_CHECK(dist_query_stride >= 0 && dist_part_stride >= 0 && label_query_stride >= 0 &&
               label_part_stride >= 0,
           MF_ERR_INVALID_ARGS, "merge strides must be non-negative");
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(part_distances, "part_distances", k_in == 0));
  MF_TRY(check_device_ptr(part_labels, "part_labels", k_in == 0));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  return launch_merge_strided(part_distances, dist_query_stride, dist_part_stride, part_labels,
                              label_query_stride, label_part_stride, nq, parts, k_in, k,
                              distances, labels, (cudaStream_t)stream);
}

int mf_kmeans_assign_workspace_size(int64_t n, int nc, int d, size_t* bytes) {
  MF_TRY(mf_flat_search_workspace_size(n, nc, d, MF_METRIC_L2, 1, bytes));
  *bytes = ((*bytes + 255) & ~size_t(255)) + (size_t)nc * d * sizeof(float);
  return MF_OK;
}

int mf_kmeans_assign(int device, void* stream, const float* x, int64_t n,
                     const float* centroids, const float* centroid_norms, int nc, int d,
                     int64_t* labels, float* min_distances, void* workspace,
                     size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, MF_METRIC_L2, 1, true));
  MF_CHECK(nc >= 1, MF_ERR_INVALID_ARGS, "need at least one centroid");
  MF_CHECK(n >= 0 && n < (1ll << 30), MF_ERR_INVALID_ARGS, "n=%lld out of range", (long long)n);
  if (n == 0) return MF_OK;
  MF_TRY(check_device_ptr(x, "x"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  MF_TRY(check_device_ptr(centroid_norms, "centroid_norms"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(min_distances, "min_distances"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  cudaStream_t s = (cudaStream_t)stream;
  const size_t flat_bytes = plan_flat(n, nc, d, 1, device).bytes;
  const size_t lo_off = (flat_bytes + 255) & ~size_t(255);
  MF_CHECK(workspace_bytes >= lo_off + (size_t)nc * d * sizeof(float), MF_ERR_INVALID_ARGS,
           "k-means assign workspace too small");
  float* cent_lo = reinterpret_cast<float*>(static_cast<char*>(workspace) + lo_off);
  const float* lo = nullptr;
  if (tc_eligible(MF_METRIC_L2, d, 1, nc)) {
    MF_TRY(launch_tf32_residual(centroids, nc, d, cent_lo, s));
    lo = cent_lo;
  }
  return run_flat_topk(device, s, x, n, centroids, centroid_norms, lo, nc, d, MF_METRIC_L2, 1,
                       nullptr, min_distances, labels, workspace, flat_bytes);
}

int mf_kmeans_update_workspace_size(int64_t n, int nc, int d, size_t* bytes) {
  clear_error();
  (void)d;
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  *bytes = kmeans_update_bytes(n, nc);
  return MF_OK;
}

int mf_kmeans_update(int device, void* stream, const float* x, int64_t n, int d,
                     const int64_t* labels, int nc, float* centroids, int64_t* counts,
                     void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_CHECK(d > 0 && nc >= 1 && n >= 0 && n < (1ll << 31) - 1, MF_ERR_INVALID_ARGS,
           "bad k-means update shape n=%lld d=%d nc=%d", (long long)n, d, nc);
  MF_TRY(check_device_ptr(x, "x", n == 0));
  MF_TRY(check_device_ptr(labels, "labels", n == 0));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  MF_TRY(check_device_ptr(counts, "counts", true));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  MF_CHECK(workspace_bytes >= kmeans_update_bytes(n, nc), MF_ERR_INVALID_ARGS,
           "k-means update workspace too small: %zu < %zu", workspace_bytes,
           kmeans_update_bytes(n, nc));
  return run_kmeans_update((cudaStream_t)stream, x, n, d, labels, nc, centroids, counts,
                           workspace, workspace_bytes);
}

int mf_kmeans_sums(int device, void* stream, const float* x, int64_t n, int d,
                   const int64_t* labels, int nc, double* sums, int64_t* counts, void* workspace,
                   size_t workspace_bytes) {
  MF_ENTER(device);
  MF_CHECK(d > 0 && nc >= 1 && n >= 0 && n < (1ll << 31) - 1, MF_ERR_INVALID_ARGS,
           "bad k-means sums shape n=%lld d=%d nc=%d", (long long)n, d, nc);
  MF_TRY(check_device_ptr(x, "x", n == 0));
  MF_TRY(check_device_ptr(labels, "labels", n == 0));
  MF_TRY(check_device_ptr(sums, "sums"));
  MF_TRY(check_device_ptr(counts, "counts"));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  MF_CHECK(workspace_bytes >= kmeans_update_bytes(n, nc), MF_ERR_INVALID_ARGS,
           "k-means sums workspace too small: %zu < %zu", workspace_bytes,
           kmeans_update_bytes(n, nc));
  return run_kmeans_update((cudaStream_t)stream, x, n, d, labels, nc, nullptr, counts, workspace,
                           workspace_bytes, sums);
}

int mf_kmeans_apply(int device, void* stream, const double* sums, const int64_t* counts, int nc,
                    int d, float* centroids) {
  MF_ENTER(device);
  MF_CHECK(d > 0 && nc >= 1, MF_ERR_INVALID_ARGS, "bad k-means apply shape d=%d nc=%d", d, nc);
  MF_TRY(check_device_ptr(sums, "sums"));
  MF_TRY(check_device_ptr(counts, "counts"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  return launch_kmeans_apply(sums, counts, nc, d, centroids, (cudaStream_t)stream);
}

int mf_ivf_add_workspace_size(int64_t n_old, int64_t n_new, int nlist, size_t* bytes) {
  clear_error();
  (void)n_old;
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  *bytes = ivf_add_bytes(n_new, nlist);
  return MF_OK;
}

int mf_ivf_add(int device, void* stream, int nlist, int d, const int64_t* old_offsets,
               const float* old_vecs, const float* old_norms, const int64_t* old_ids,
               int64_t n_old, const float* new_vecs, const float* new_norms,
               const int64_t* new_ids, const int64_t* new_labels, int64_t n_new,
               int64_t* out_offsets, float* out_vecs, float* out_norms, int64_t* out_ids,
               void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_CHECK(nlist >= 1 && d > 0 && d % 4 == 0, MF_ERR_INVALID_ARGS, "nlist=%d d=%d", nlist, d);
  MF_CHECK(n_old >= 0 && n_new >= 0 && n_new < (1ll << 31) - 1, MF_ERR_INVALID_ARGS,
           "bad row counts");
  if (n_old > 0) {
    MF_TRY(check_device_ptr(old_offsets, "old_offsets"));
    MF_TRY(check_device_ptr(old_vecs, "old_vecs"));
    MF_TRY(check_device_ptr(old_norms, "old_norms"));
    MF_TRY(check_device_ptr(old_ids, "old_ids"));
  }
  if (n_new > 0) {
    MF_TRY(check_device_ptr(new_vecs, "new_vecs"));
    MF_TRY(check_device_ptr(new_norms, "new_norms"));
    MF_TRY(check_device_ptr(new_ids, "new_ids"));
    MF_TRY(check_device_ptr(new_labels, "new_labels"));
  }
  MF_TRY(check_device_ptr(out_offsets, "out_offsets"));
  if (n_old + n_new > 0) {
    MF_TRY(check_device_ptr(out_vecs, "out_vecs"));
    MF_TRY(check_device_ptr(out_norms, "out_norms"));
    MF_TRY(check_device_ptr(out_ids, "out_ids"));
  }
  MF_TRY(check_device_ptr(workspace, "workspace"));
  MF_CHECK(workspace_bytes >= ivf_add_bytes(n_new, nlist), MF_ERR_INVALID_ARGS,
           "ivf add workspace too small");
  return run_ivf_add((cudaStream_t)stream, nlist, d, old_offsets, old_vecs, old_norms, old_ids,
                     n_old, new_vecs, new_norms, new_ids, new_labels, n_new, out_offsets,
                     out_vecs, out_norms, out_ids, workspace, workspace_bytes);
}

// ------------------------------------------------------------ range search
int mf_flat_range_workspace_size(int64_t nq, int64_t nb, int d, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  int dev = 0;
  cudaGetDevice(&dev);
  FlatPlan p = plan_flat(nq, nb, d, 32, dev, 32, false);
  Carver c(nullptr, 0);
  c.take<float>(nq);
  c.take<int>(1);
  c.take<int64_t>((size_t)nq * p.splits);
  c.take<int64_t>((size_t)nq * p.splits + 1);
  *bytes = c.used;
  return MF_OK;
}

namespace {
struct FlatRangeWs {
  FlatPlan p;
  float* qn;
  int* counter;
  int64_t* counts;
  int64_t* offsets;
};
int carve_flat_range(FlatRangeWs& w, int64_t nq, int64_t nb, int d, int device, void* ws,
                     size_t bytes) {
  w.p = plan_flat(nq, nb, d, 32, device, 32, false);
  Carver c(ws, bytes);
  w.qn = c.take<float>(nq);
  w.counter = c.take<int>(1);
  w.counts = c.take<int64_t>((size_t)nq * w.p.splits);
  w.offsets = c.take<int64_t>((size_t)nq * w.p.splits + 1);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "range workspace too small: %zu < %zu", bytes, c.used);
  return MF_OK;
}
ScanArgs flat_range_args(const FlatRangeWs& w, const float* xq, int64_t nq, const float* xb,
                         const float* xb_norms, int64_t nb, int d, float radius) {
  ScanArgs a{};
  a.xq = xq;
  a.qnorms = w.qn;
  a.xb = xb;
  a.xnorms = xb_norms;
  a.d = d;
  a.k = 1;
  a.nq = nq;
  a.P = w.p.splits;
  a.flat = 1;
  a.nqt = w.p.nqt;
  a.nb = nb;
  a.rows_per_split = w.p.rows_per_split;
  a.counter = w.counter;
  a.radius = radius;
  a.counts = w.counts;
  a.offsets = w.offsets;
  return a;
}
int read_total(const int64_t* dev_total, int64_t* total, cudaStream_t s) {
  MF_CUDA(cudaMemcpyAsync(total, dev_total, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  MF_CUDA(cudaStreamSynchronize(s));
  return MF_OK;
}
}  // namespace

int mf_flat_range_count(int device, void* stream, const float* xq, int64_t nq, const float* xb,
                        const float* xb_norms, int64_t nb, int d, int metric, float radius,
                        int64_t* lims, int64_t* total, void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, 1, false));
  MF_CHECK(total != nullptr, MF_ERR_INVALID_ARGS, "total is NULL");
  MF_CHECK(nb < (1ll << 31) - 1 && nq >= 0, MF_ERR_INVALID_ARGS, "bad sizes");
  MF_TRY(check_device_ptr(lims, "lims"));
  *total = 0;
  cudaStream_t s = (cudaStream_t)stream;
  if (nq == 0) {
    MF_CUDA(cudaMemsetAsync(lims, 0, sizeof(int64_t), s));
    return MF_OK;
  }
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  if (metric == MF_METRIC_L2) MF_TRY(check_device_ptr(xb_norms, "xb_norms", nb == 0));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  FlatRangeWs w;
  MF_TRY(carve_flat_range(w, nq, nb, d, device, workspace, workspace_bytes));
  if (metric == MF_METRIC_L2) MF_TRY(launch_norms(xq, nq, d, w.qn, s));
  MF_CUDA(cudaMemsetAsync(w.counts, 0, sizeof(int64_t) * nq * w.p.splits, s));
  ScanArgs a = flat_range_args(w, xq, nq, xb, xb_norms, nb, d, radius);
  if (nb > 0) MF_TRY(launch_scan(a, metric, kEpiCount, (int64_t)w.p.nqt * w.p.splits, device, s));
  MF_TRY(launch_exclusive_scan_i64(w.counts, nq * w.p.splits, w.offsets, s));
  MF_TRY(launch_lims(w.offsets, nq, w.p.splits, lims, s));
  return read_total(w.offsets + nq * w.p.splits, total, s);
}

int mf_flat_range_fill(int device, void* stream, const float* xq, int64_t nq, const float* xb,
                       const float* xb_norms, int64_t nb, int d, int metric, float radius,
                       const int64_t* ids, const int64_t* lims, float* distances,
                       int64_t* labels, void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, 1, false));
  (void)lims;
  if (nq == 0 || nb == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(xb, "xb"));
  MF_TRY(check_device_ptr(ids, "ids", true));
  MF_TRY(check_device_ptr(distances, "distances", true));
  MF_TRY(check_device_ptr(labels, "labels", true));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  FlatRangeWs w;
  MF_TRY(carve_flat_range(w, nq, nb, d, device, workspace, workspace_bytes));
  ScanArgs a = flat_range_args(w, xq, nq, xb, xb_norms, nb, d, radius);
  a.ids = ids;
  a.out_d = distances;
  a.out_l = labels;
  return launch_scan(a, metric, kEpiFill, (int64_t)w.p.nqt * w.p.splits, device,
                     (cudaStream_t)stream);
}

int mf_ivf_range_workspace_size(int64_t nq, int nlist, int nprobe, int d, size_t* bytes) {
  clear_error();
  MF_CHECK(bytes != nullptr, MF_ERR_INVALID_ARGS, "bytes is NULL");
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  int dev = 0;
  cudaGetDevice(&dev);
  Carver c(nullptr, 0);
  carve_ivf(c, nq, nlist, effective_nprobe(nprobe, nlist), d, 1, 2, dev);
  *bytes = c.used;
  return MF_OK;
}

namespace {
ScanArgs ivf_range_args(const IvfWs& w, const float* xq, int64_t nq, int P,
                        const int64_t* list_offsets, const float* list_vecs,
                        const float* list_norms, int d, float radius) {
  ScanArgs a{};
  a.xq = xq;
  a.qnorms = w.qn;
  a.xb = list_vecs;
  a.xnorms = list_norms;
  a.d = d;
  a.k = 1;
  a.nq = nq;
  a.P = P;
  a.flat = 0;
  a.items = w.g.items;
  a.item_total = w.g.item_total;
  a.list_offsets = list_offsets;
  a.pair_offsets = w.g.pair_offsets;
  a.pairs = w.g.pairs;
  a.counter = w.g.counter;
  a.radius = radius;
  a.counts = w.pair_counts;
  a.offsets = w.pair_offsets64;
  return a;
}
}  // namespace

int mf_ivf_range_count(int device, void* stream, const float* xq, int64_t nq,
                       const float* centroids, const float* centroid_norms, int nlist,
                       int nprobe, const int64_t* list_offsets, const float* list_vecs,
                       const float* list_norms, int d, int metric, float radius, int64_t* lims,
                       int64_t* total, void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, 1, false));
  MF_CHECK(total != nullptr, MF_ERR_INVALID_ARGS, "total is NULL");
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  const int P = effective_nprobe(nprobe, nlist);
  MF_CHECK(P <= kMaxK, MF_ERR_INVALID_ARGS, "nprobe=%d exceeds %d", P, kMaxK);
  MF_CHECK(nq >= 0 && nq * P < (1ll << 31), MF_ERR_INVALID_ARGS, "nq*nprobe too large");
  MF_TRY(check_device_ptr(lims, "lims"));
  *total = 0;
  cudaStream_t s = (cudaStream_t)stream;
  if (nq == 0) {
    MF_CUDA(cudaMemsetAsync(lims, 0, sizeof(int64_t), s));
    return MF_OK;
  }
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(centroids, "centroids"));
  MF_TRY(check_device_ptr(centroid_norms, "centroid_norms", coarse_metric(metric) != MF_METRIC_L2));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, nullptr, nullptr, metric));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, P, d, 1, 2, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "IVF range workspace too small");
  MF_TRY(run_flat_topk(device, s, xq, nq, centroids, centroid_norms, nullptr, nlist, d,
                       coarse_metric(metric), P, nullptr, w.coarse_d, w.coarse_l, w.flat_ws,
                       w.flat_bytes));
  if (metric == MF_METRIC_L2) MF_TRY(launch_norms(xq, nq, d, w.qn, s));
  MF_TRY(run_ivf_groups_ex(w.g, w.coarse_l, nq, P, nlist, list_offsets, nullptr, nullptr,
                           nullptr, 0, w.pair_counts, kScanTQ, s));
  ScanArgs a = ivf_range_args(w, xq, nq, P, list_offsets, list_vecs, list_norms, d, radius);
  MF_TRY(launch_scan(a, metric, kEpiCount, nq * P, device, s));
  MF_TRY(launch_exclusive_scan_i64(w.pair_counts, nq * P, w.pair_offsets64, s));
  MF_TRY(launch_lims(w.pair_offsets64, nq, P, lims, s));
  return read_total(w.pair_offsets64 + nq * P, total, s);
}

int mf_ivf_range_fill(int device, void* stream, const float* xq, int64_t nq,
                      const float* centroids, const float* centroid_norms, int nlist, int nprobe,
                      const int64_t* list_offsets, const float* list_vecs,
                      const float* list_norms, const int64_t* list_ids, int d, int metric,
                      float radius, const int64_t* lims, float* distances, int64_t* labels,
                      void* workspace, size_t workspace_bytes) {
  MF_ENTER(device);
  MF_TRY(check_common(d, metric, 1, false));
  (void)centroids;
  (void)centroid_norms;
  (void)lims;
  MF_CHECK(nlist >= 1 && nprobe >= 1, MF_ERR_INVALID_ARGS, "nlist=%d nprobe=%d", nlist, nprobe);
  const int P = effective_nprobe(nprobe, nlist);
  if (nq == 0) return MF_OK;
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_ivf_lists(list_offsets, list_vecs, list_norms, list_ids, nullptr, metric));
  MF_TRY(check_device_ptr(distances, "distances", true));
  MF_TRY(check_device_ptr(labels, "labels", true));
  MF_TRY(check_device_ptr(workspace, "workspace"));
  Carver c(workspace, workspace_bytes);
  IvfWs w = carve_ivf(c, nq, nlist, P, d, 1, 2, device);
  MF_CHECK(c.fits(), MF_ERR_INVALID_ARGS, "IVF range workspace too small");
  ScanArgs a = ivf_range_args(w, xq, nq, P, list_offsets, list_vecs, list_norms, d, radius);
  a.ids = list_ids;
  a.out_d = distances;
  a.out_l = labels;
  return launch_scan(a, metric, kEpiFill, nq * P, device, (cudaStream_t)stream);
}

int mf_tf32_residual(int device, void* stream, const float* x, int64_t n, int d, float* lo) {
  MF_ENTER(device);
  MF_CHECK(n >= 0 && d > 0 && d % 4 == 0, MF_ERR_INVALID_ARGS, "bad shape n=%lld d=%d",
           (long long)n, d);
  if (n == 0) return MF_OK;
  MF_TRY(check_device_ptr(x, "x"));
  MF_TRY(check_device_ptr(lo, "lo"));
  return launch_tf32_residual(x, n, d, lo, (cudaStream_t)stream);
}

int mf_set_filter_small_group(int queries) {
  clear_error();
  MF_CHECK(queries >= 0 && queries <= few_max_queries(), MF_ERR_INVALID_ARGS,
           "queries=%d (0 to %d)", queries, few_max_queries());
  g_filter_small_group = queries;
  return MF_OK;
}

int mf_set_filter_groups(int groups) {
  clear_error();
  MF_CHECK(groups == 1 || groups == 2, MF_ERR_INVALID_ARGS, "groups=%d (1 or 2)", groups);
  set_filter_groups(groups);
  return MF_OK;
}

int mf_set_scan_engine(int engine) {
  clear_error();
  MF_CHECK(engine >= 0 && engine <= 3, MF_ERR_INVALID_ARGS, "engine %d not in {0,1,2,3}", engine);
  set_scan_engine(engine);
  return MF_OK;
}

int mf_device_error(int device, int* code) {
  MF_ENTER(device);
  MF_CHECK(code != nullptr, MF_ERR_INVALID_ARGS, "code is NULL");
  MF_CUDA(cudaDeviceSynchronize());
  int v = 0;
  MF_TRY(read_device_error(&v));
  *code = v ? MF_ERR_TIMEOUT : MF_OK;
  return MF_OK;
}

}  // extern "C"
