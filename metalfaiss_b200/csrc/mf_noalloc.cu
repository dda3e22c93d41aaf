// Flat k-NN search for callers that cannot allocate device memory.
//
// mf_flat_search needs a caller-provided workspace. Some callers have no way
// to get one: a host runtime that hands this library only the buffers it
// already owns (a plugin or FFI binding with no device allocator of its own),
// code that runs where cudaMalloc is not allowed or would stall other work
// on the device, or a process that must keep its device footprint fixed after
// start-up. mf_flat_search_noalloc serves them. Its scratch is one fixed
// array of kNoAllocScratchBytes in this library's device image. Every GPU
// that loads the library holds that array until the process exits.
//
// Contract:
//  * Every call looks up the array's device address on `device` (with that
//    device current). The address is not cached: a cached one would outlive
//    a device reset or a released primary context and point at memory this
//    library no longer owns. The lookup is cheap next to a search, but the
//    first one on a device may load this library's device image there, so
//    make the first call on a device before any stream capture starts on it.
//  * A search whose scratch need exceeds kNoAllocScratchBytes is rejected
//    with MF_ERR_INVALID_ARGS before anything is launched.
//  * No call allocates or frees device memory.
//  * Every call on a device shares the one array, and the array keeps the
//    previous call's contents. The search clears what must start at zero
//    (its work counter) on the stream before the scan reads it. Two calls
//    whose work overlaps on the GPU (different streams, or different host
//    threads) race on the array and give wrong results: serialize them.
#include "mf_scan.cuh"

namespace mf {
namespace {

// 16 MiB: query norms + per-split partial top-k + the query tf32 residuals
// (mf_flat_search_workspace_size gives the need of one search). On a 148-SM
// B200, nq=1024, d=128, k=10 needs about 4.8 MiB at any nb, and nq=4096,
// d=512, k=10 about 12.7 MiB; nq=4096, d=128, k=256 needs about 122 MiB and
// is rejected.
constexpr size_t kNoAllocScratchBytes = static_cast<size_t>(MF_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch in the current context (the caller has
// made `device` current). In host code g_noalloc_scratch names only a host
// stand-in for the device symbol, so its address must come from the runtime.
int noalloc_scratch(void** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(static scratch)");
  MF_CHECK(p != nullptr && (reinterpret_cast<uintptr_t>(p) & 255) == 0, MF_ERR_CUDA,
           "static scratch address %p is not 256-byte aligned", p);
  *out = p;
  return MF_OK;
}

}  // namespace
}  // namespace mf

using namespace mf;

extern "C" {

int mf_flat_search_noalloc(int device, void* stream, const float* xq, int64_t nq,
                           const float* xb, const float* xb_norms, const float* xb_lo,
                           int64_t nb, int d, int metric, int k, const int64_t* ids,
                           float* distances, int64_t* labels) {
  clear_error();
  DeviceGuard guard(device);
  if (guard.status != MF_OK) return guard.status;
  MF_CHECK(d > 0 && d % 4 == 0, MF_ERR_INVALID_ARGS,
           "d=%d must be a positive multiple of 4 (pad rows with zeros)", d);
  MF_CHECK(metric >= 0 && metric <= 3, MF_ERR_METRIC,
           "metric %d is not one of INNER_PRODUCT(0), L2(1), L1(2), LINF(3)", metric);
  MF_CHECK(k >= 1 && k <= kMaxK, MF_ERR_INVALID_ARGS, "k=%d must be in [1, %d]", k, kMaxK);
  MF_CHECK(nq >= 0 && nb >= 0, MF_ERR_INVALID_ARGS, "negative sizes");
  MF_CHECK(nb < (1ll << 31) - 1, MF_ERR_INVALID_ARGS, "nb=%lld exceeds 2^31-2 rows per call",
           (long long)nb);
  MF_CHECK(nq < (1ll << 31) / 2, MF_ERR_INVALID_ARGS, "nq too large");
  if (nq == 0) return MF_OK;
  // the fused top-k's scratch: the distance-matrix path is taken only when
  // the scratch also holds the matrix
  const size_t need = plan_flat(nq, nb, d, k, device).bytes_min;
  MF_CHECK(need <= kNoAllocScratchBytes, MF_ERR_INVALID_ARGS,
           "flat search of nq=%lld nb=%lld d=%d k=%d needs %zu bytes of scratch; the static "
           "scratch holds %zu (split the queries, or call mf_flat_search with a workspace)",
           (long long)nq, (long long)nb, d, k, need, kNoAllocScratchBytes);
  MF_TRY(check_device_ptr(xq, "xq"));
  MF_TRY(check_device_ptr(distances, "distances"));
  MF_TRY(check_device_ptr(labels, "labels"));
  MF_TRY(check_device_ptr(xb, "xb", nb == 0));
  MF_TRY(check_device_ptr(ids, "ids", true));
  if (metric == MF_METRIC_L2) MF_TRY(check_device_ptr(xb_norms, "xb_norms", nb == 0));
  MF_TRY(check_device_ptr(xb_lo, "xb_lo", true));
  void* scratch = nullptr;
  MF_TRY(noalloc_scratch(&scratch));
  return run_flat_topk(device, (cudaStream_t)stream, xq, nq, xb, xb_norms, xb_lo, nb, d, metric,
                       k, ids, distances, labels, scratch, kNoAllocScratchBytes);
}

}  // extern "C"
