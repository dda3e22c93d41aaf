// Optional per-kernel CUDA-event timing of the launches this library makes.
// When enabled, every tracked launch is bracketed by two events recorded on
// the launching stream; totals are read after the caller synchronizes.
#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "mf_timing.cuh"

namespace mf {
namespace {
struct Rec {
  std::string name;
  cudaEvent_t a, b;
};
std::mutex g_mu;
bool g_on = false;
std::vector<Rec> g_recs;
}  // namespace

std::atomic<long long> g_launches{0};

bool timing_enabled() { return g_on; }
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void* timing_begin(const char* name, cudaStream_t s) {
  if (!g_on) return nullptr;
  Rec* r = new Rec{name, nullptr, nullptr};
  if (cudaEventCreate(&r->a) != cudaSuccess || cudaEventCreate(&r->b) != cudaSuccess) {
    delete r;
    return nullptr;
  }
  cudaEventRecord(r->a, s);
  return r;
}

void timing_end(void* h, cudaStream_t s) {
  if (!h) return;
  Rec* r = static_cast<Rec*>(h);
  cudaEventRecord(r->b, s);
  std::lock_guard<std::mutex> lk(g_mu);
  g_recs.push_back(*r);
  delete r;
}

}  // namespace mf

using namespace mf;

extern "C" {

int mf_timing_enable(int enable) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_on = enable != 0;
  return MF_OK;
}

int mf_timing_reset(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& r : g_recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  g_recs.clear();
  return MF_OK;
}

int64_t mf_launch_count(void) { return g_launches.load(); }

int mf_timing_read(const char* kernel, double* total_ms, int64_t* launches) {
  if (!kernel || !total_ms || !launches) return fail(MF_ERR_INVALID_ARGS, "NULL argument");
  std::lock_guard<std::mutex> lk(g_mu);
  double t = 0.0;
  int64_t n = 0;
  for (auto& r : g_recs) {
    if (r.name != kernel) continue;
    float ms = 0.f;
    cudaError_t e = cudaEventElapsedTime(&ms, r.a, r.b);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime (synchronize first)");
    t += ms;
    ++n;
  }
  *total_ms = t;
  *launches = n;
  return MF_OK;
}

}  // extern "C"
