// Minimal C++ emulation of the Metal Shading Language subset used by the
// reference's compute kernels: address-space qualifiers, uint, thread
// position built-ins and threadgroup_barrier. Threadgroup arrays become
// function statics shared by the emulated threads of the running group
// (groups run one after another).
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>

struct msl_uint3 {
  unsigned x, y, z;
};
extern thread_local msl_uint3 thread_position_in_threadgroup;
extern thread_local msl_uint3 threads_per_threadgroup;
extern thread_local msl_uint3 threadgroup_position_in_grid;
extern thread_local msl_uint3 thread_position_in_grid;
extern thread_local msl_uint3 threads_per_grid;
extern thread_local msl_uint3 threadgroups_per_grid;

namespace mem_flags {
enum flags { mem_none = 0, mem_device = 1, mem_threadgroup = 2, mem_texture = 4 };
}
void threadgroup_barrier(int flags);
void msl_launch(unsigned grid_x, unsigned tg_x, void (*fn)(void*), void* ctx);

typedef unsigned int uint;
using std::abs;
using std::fabs;
using std::fma;
using std::max;
using std::min;

#define thread
#define device
#define constant const
#define threadgroup static
