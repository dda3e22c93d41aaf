// Shared helpers of the sm_100a kernels: status/error plumbing, keys for the
// fused top-k, cp.async wrappers and the per-device launch facts.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/metalfaiss_b200.h"

namespace mf {

// ------------------------------------------------------------------ errors
// Sets the thread-local last-error message and returns `code`.
int fail(int code, const char* fmt, ...);
// Maps a CUDA error to MF_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t e, const char* what);
void clear_error();

#define MF_CUDA(call)                                   \
  do {                                                  \
    cudaError_t _e = (call);                            \
    if (_e != cudaSuccess) return ::mf::cuda_fail(_e, #call); \
  } while (0)

// Checks the launch just made and counts it (mf_launch_count).
void count_launch();
#define MF_LAUNCH_CHECK()                                              \
  do {                                                                 \
    cudaError_t _e = cudaGetLastError();                               \
    if (_e != cudaSuccess) return ::mf::cuda_fail(_e, "kernel launch"); \
    ::mf::count_launch();                                              \
  } while (0)

#define MF_CHECK(cond, code, ...)                 \
  do {                                            \
    if (!(cond)) return ::mf::fail(code, __VA_ARGS__); \
  } while (0)

#define MF_TRY(call)            \
  do {                          \
    int _s = (call);            \
    if (_s != MF_OK) return _s; \
  } while (0)

// Makes `device` current for the lifetime of the guard and restores the
// caller's device afterwards.
struct DeviceGuard {
  int prev = -1;
  int status = MF_OK;
  explicit DeviceGuard(int device);
  ~DeviceGuard();
};

// Rejects host pointers and misaligned pointers before any kernel sees them.
int check_device_ptr(const void* p, const char* name, bool allow_null = false);
int num_sms(int device);

// Carves sub-buffers out of a caller workspace (256-byte aligned pieces).
struct Carver {
  char* base;
  size_t cap;
  size_t used = 0;
  Carver(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <class T>
  T* take(size_t count) {
    used = (used + 255) & ~size_t(255);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * sizeof(T);
    return p;
  }
  bool fits() const { return used <= cap; }
};

// ---------------------------------------------------------------- top-k keys
// A candidate is one 64-bit key: the order-preserving image of its fp32
// distance in the high word and a unique 32-bit index in the low word, so
// unsigned comparison ranks by (distance, index) and every key is distinct.
constexpr unsigned long long kEmptyKey = ~0ull;

__device__ __forceinline__ unsigned int float_to_ordered(float f) {
  unsigned int u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(unsigned int o) {
  unsigned int u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}
__device__ __forceinline__ unsigned long long make_key(float dist, unsigned int idx) {
  return (static_cast<unsigned long long>(float_to_ordered(dist)) << 32) | idx;
}
// The largest key with distance <= d: every candidate at distance d passes a
// `key < bound` test except the (impossible) index 0xffffffff.
__device__ __forceinline__ unsigned long long bound_key(float d) {
  return (d != d || d == __int_as_float(0x7f800000)) ? kEmptyKey : make_key(d, 0xffffffffu);
}
__device__ __forceinline__ float key_dist(unsigned long long key) {
  return ordered_to_float(static_cast<unsigned int>(key >> 32));
}
__device__ __forceinline__ unsigned int key_index(unsigned long long key) {
  return static_cast<unsigned int>(key & 0xffffffffull);
}

// -------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src, bool valid) {
  unsigned int dst = static_cast<unsigned int>(__cvta_generic_to_shared(smem_dst));
  int src_bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(gmem_src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ unsigned int lanemask_lt() {
  unsigned int m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Distance epilogues shared by every kernel. L2 mirrors the reference's
// (||q||^2 + ||x||^2) - (q.x + q.x) clamped at zero (python/metalfaiss/distances.py:170-173);
// inner product is negated (python/metalfaiss/indexflat.py:93).
__device__ __forceinline__ float l2_from_dot(float qn, float xn, float dot) {
  float d = __fsub_rn(__fadd_rn(qn, xn), __fadd_rn(dot, dot));
  return fmaxf(d, 0.0f) + 0.0f;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace mf
