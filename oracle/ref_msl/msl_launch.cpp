// Launcher for msl_shim.h: one OS thread per emulated Metal thread, one
// std::barrier per threadgroup, threadgroups run in order.
#include <barrier>
#include <thread>
#include <vector>

struct msl_uint3 {
  unsigned x, y, z;
};
thread_local msl_uint3 thread_position_in_threadgroup;
thread_local msl_uint3 threads_per_threadgroup;
thread_local msl_uint3 threadgroup_position_in_grid;
thread_local msl_uint3 thread_position_in_grid;
thread_local msl_uint3 threads_per_grid;
thread_local msl_uint3 threadgroups_per_grid;

static std::barrier<>* g_barrier = nullptr;

void threadgroup_barrier(int) { g_barrier->arrive_and_wait(); }

void msl_launch(unsigned grid_x, unsigned tg_x, void (*fn)(void*), void* ctx) {
  if (grid_x == 0 || tg_x == 0) return;
  const unsigned groups = (grid_x + tg_x - 1) / tg_x;
  for (unsigned g = 0; g < groups; ++g) {
    const unsigned size = std::min(tg_x, grid_x - g * tg_x);
    std::barrier<> bar(size);
    g_barrier = &bar;
    std::vector<std::thread> ts;
    ts.reserve(size);
    for (unsigned t = 0; t < size; ++t) {
      ts.emplace_back([=]() {
        thread_position_in_threadgroup = {t, 0, 0};
        threads_per_threadgroup = {size, 1, 1};
        threadgroup_position_in_grid = {g, 0, 0};
        thread_position_in_grid = {g * tg_x + t, 0, 0};
        threads_per_grid = {grid_x, 1, 1};
        threadgroups_per_grid = {groups, 1, 1};
        fn(ctx);
      });
    }
    for (auto& th : ts) th.join();
    g_barrier = nullptr;
  }
}
