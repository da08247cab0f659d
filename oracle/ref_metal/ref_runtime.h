// ref_runtime.h — runs Metal compute dispatches of the reference's kernels on the host. TEST INFRASTRUCTURE ONLY.
//
// One threadgroup at a time per OS thread: its threads are cooperative fibers (ucontext) that run until they reach a
// collective (a SIMD-group function, a simdgroup matrix product or threadgroup_barrier) or return. When every fiber
// is waiting or done, the scheduler resolves the collectives whose SIMD group has fully arrived (a lane that
// returned or waits at a barrier does not take part, as inactive lanes on the GPU), or, when every live fiber waits
// at the barrier, releases the barrier. Threadgroups of one dispatch run in parallel over OpenMP threads, each with
// its own fibers and its own `static thread_local` threadgroup arrays.
#pragma once

#include <cstdint>

namespace refrt {

struct Ctx {
    uint32_t tg[3];   // threadgroup_position_in_grid
    uint32_t ng[3];   // threadgroups_per_grid
    uint32_t tp[3];   // thread_position_in_threadgroup
    uint32_t tid;     // thread_index_in_threadgroup
    uint32_t sid;     // simdgroup_index_in_threadgroup
    uint32_t lane;    // thread_index_in_simdgroup
    uint32_t gid[3];  // thread_position_in_grid
};

typedef void (*Body)(void* user, const Ctx& c);

// Runs grid[0] x grid[1] x grid[2] threadgroups of tpg[0] x tpg[1] x tpg[2] threads (at most 1024), calling
// body(user, ctx) once per thread. Aborts the process with a message on a collective that cannot complete.
void dispatch(const uint32_t grid[3], const uint32_t tpg[3], Body body, void* user);

template <class F>
inline void run(uint32_t gx, uint32_t gy, uint32_t gz, uint32_t tx, uint32_t ty, uint32_t tz, F&& f) {
    const uint32_t g[3] = {gx, gy, gz}, t[3] = {tx, ty, tz};
    dispatch(g, t, [](void* u, const Ctx& c) { (*(F*)u)(c); }, (void*)&f);
}

}  // namespace refrt
